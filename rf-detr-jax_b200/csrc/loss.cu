// Set-prediction losses of one decoder layer for sm_100a, with their gradients.
//
// Reference (src/rfdetr_jax/models/criterion.py):
//   loss_labels, IA-BCE (:157-208): with p = sigmoid(x), matched (image, query, class) entries
//     carry pos = w, neg = 1 - w, where w = clip(p_m^alpha * iou^(1-alpha), 0.01) is
//     stop-gradient (iou of the stop-gradient predicted box and the target box,
//     box_ops.py:78-91); every other entry carries pos = 0, neg = p^2 (differentiated);
//     loss = sum(neg * x - log_sigmoid(x) * (pos + neg)) / num_boxes;
//   loss_boxes (:233-250): L1 and 1 - GIoU (box_ops.py:94-103) over valid matched pairs, each
//     divided by num_boxes.
// Per entry the IA-BCE term and its derivative have closed forms, with softplus(x) = x -
// log_sigmoid(x):
//   unmatched: p^2 softplus(x)                    d/dx = p^3 + 2 p^2 (1 - p) softplus(x)
//   matched:   (1 - w) x + softplus(-x)           d/dx = p - w
// With ia_bce off the reference uses the sigmoid focal loss with gamma = 2 (:210-224; its
// mean over queries times the query count is a plain sum), alpha_t = alpha / 1 - alpha for
// matched / unmatched entries (1 when alpha < 0):
//   unmatched: a0 p^2 softplus(x)                 d/dx = a0 (p^3 + 2 p^2 (1 - p) softplus(x))
//   matched:   a1 (1 - p)^2 softplus(-x)          d/dx = -a1 (1 - p)^2 (2 p softplus(-x) + 1 - p)
// The kernel writes the three loss values and the gradients for unit cotangents: dloss_ce/dx
// ([B, Q, C]) and the L1 and GIoU gradients with respect to the predicted boxes ([B, Q, 4]).
//
// One CTA per (layer, image, tile of kLossRows queries), one launch for every layer.  The CTA
// first evaluates all of its tile's (query, class) entries as unmatched, with 16-byte loads all
// issued before the arithmetic (the tile is one contiguous run of logits), then scans the
// image's matcher slots for the valid ones whose query falls in its tile (a query is matched at
// most once: groups own disjoint query ranges); a tile of 96 queries amortises that scan, which
// every CTA of the image repeats, better than 32 or 64 (27 / 29 / 36 µs for three config-4
// layers at 96 / 64 / 32).  For those it computes the box losses and
// gradients and the IA-BCE weight, overwrites the matched entry's gradient (after a barrier, so
// the dense write is ordered before it) and adds the difference between the matched and the
// unmatched value to the loss partial.  Loss partials are summed across CTAs with float atomics.
#include <algorithm>

#include "common.cuh"

namespace rfdetr {
namespace {

constexpr int kLossThreads = 256;
constexpr int kLossRows = 96;

constexpr int kLossVecs = 3;    // float4 loads a thread keeps in flight in the dense pass
constexpr int kSlotUnroll = 4;  // matcher slots a thread reads at once

// log(1 + e) for e in [0, 1]: 2 atanh(t) with t = e / (2 + e) in [0, 1/3], by its odd series
// t + t^3/3 + ... + t^15/15 (truncation below 2e-9 relative at t = 1/3).
__device__ __forceinline__ float log1p_unit(float e) {
    const float t = __fdividef(e, 2.f + e);
    const float t2 = t * t;
    float s = 1.f / 15.f;
    s = fmaf(s, t2, 1.f / 13.f);
    s = fmaf(s, t2, 1.f / 11.f);
    s = fmaf(s, t2, 1.f / 9.f);
    s = fmaf(s, t2, 1.f / 7.f);
    s = fmaf(s, t2, 1.f / 5.f);
    s = fmaf(s, t2, 1.f / 3.f);
    s = fmaf(s, t2, 1.f);
    return 2.f * t * s;
}

// sigmoid(x), 1 - sigmoid(x) and softplus(x) from one exponential (no cancellation in 1 - p).
struct Logistic {
    float p, q, sp;
};
__device__ __forceinline__ Logistic logistic(float x) {
    const float e = __expf(-fabsf(x));
    const float r = __fdividef(1.f, 1.f + e);
    const bool pos = x >= 0.f;
    return {pos ? r : e * r, pos ? e * r : r, fmaxf(x, 0.f) + log1p_unit(e)};
}

// Value and d/dx of one unmatched entry: a0 p^2 softplus(x).
__device__ __forceinline__ float2 unmatched_term(float x, float a0) {
    const Logistic l = logistic(x);
    const float pp = l.p * l.p;
    return make_float2(a0 * pp * l.sp, a0 * pp * (l.p + 2.f * l.q * l.sp));
}

// Value and d/dx of one matched entry: IA-BCE with weight w, or focal with alpha_t a1.
__device__ __forceinline__ float2 matched_term(float x, bool ia_bce, float w, float a1) {
    const Logistic l = logistic(x);
    const float spn = l.sp - x;  // softplus(-x)
    if (ia_bce) return make_float2((1.f - w) * x + spn, l.p - w);
    const float qq = l.q * l.q;
    return make_float2(a1 * qq * spn, -a1 * qq * (2.f * l.p * spn + l.q));
}

struct Box {
    float x0, y0, x1, y1;
};

// box_ops.py:27-32 (cxcywh -> xyxy, negative sizes clamped to zero).
__device__ __forceinline__ Box to_xyxy(const float *b) {
    const float w = fmaxf(b[2], 0.f), h = fmaxf(b[3], 0.f);
    return {b[0] - 0.5f * w, b[1] - 0.5f * h, b[0] + 0.5f * w, b[1] + 0.5f * h};
}

__device__ __forceinline__ float iou_of(const Box &a, const Box &b) {
    const float area1 = (a.x1 - a.x0) * (a.y1 - a.y0), area2 = (b.x1 - b.x0) * (b.y1 - b.y0);
    const float iw = fmaxf(fminf(a.x1, b.x1) - fmaxf(a.x0, b.x0), 0.f);
    const float ih = fmaxf(fminf(a.y1, b.y1) - fmaxf(a.y0, b.y0), 0.f);
    const float inter = iw * ih;
    const float uni = area1 + area2 - inter;
    return inter / fmaxf(uni, 1e-7f);
}

// 1 - GIoU of predicted cxcywh box s against target t, and its gradient with respect to s
// scaled by `scale` (box_ops.py:78-103 differentiated by hand; ties of min/max are measure-zero
// and follow the strict comparisons below).
__device__ void giou_loss_grad(const float *s, const float *t, float scale, float &loss, float *grad) {
    const float wp = fmaxf(s[2], 0.f), hp = fmaxf(s[3], 0.f);
    const float a0 = s[0] - 0.5f * wp, a1 = s[1] - 0.5f * hp, a2 = s[0] + 0.5f * wp, a3 = s[1] + 0.5f * hp;
    const Box b = to_xyxy(t);
    const float area1 = (a2 - a0) * (a3 - a1), area2 = (b.x1 - b.x0) * (b.y1 - b.y0);
    const float ltx = fmaxf(a0, b.x0), lty = fmaxf(a1, b.y0), rbx = fminf(a2, b.x1), rby = fminf(a3, b.y1);
    const float iwr = rbx - ltx, ihr = rby - lty;
    const float iw = fmaxf(iwr, 0.f), ih = fmaxf(ihr, 0.f);
    const float inter = iw * ih;
    const float uni = area1 + area2 - inter;
    const float U = fmaxf(uni, 1e-7f);
    const float iou = inter / U;
    const float eltx = fminf(a0, b.x0), elty = fminf(a1, b.y0), erbx = fmaxf(a2, b.x1), erby = fmaxf(a3, b.y1);
    const float ewr = erbx - eltx, ehr = erby - elty;
    const float ew = fmaxf(ewr, 0.f), eh = fmaxf(ehr, 0.f);
    const float area = ew * eh;
    const float A = fmaxf(area, 1e-7f);
    const float giou = iou - (area - uni) / A;
    loss = 1.f - giou;

    const float d_giou = -scale;
    const float d_iou = d_giou;
    float d_uni = d_giou / A;
    float d_area = -d_giou / A + (area > 1e-7f ? d_giou * (area - uni) / (A * A) : 0.f);
    float d_inter = d_iou / U;
    if (uni > 1e-7f) d_uni += -d_iou * inter / (U * U);
    const float d_area1 = d_uni;
    d_inter -= d_uni;
    const float d_iwr = iwr > 0.f ? d_inter * ih : 0.f;
    const float d_ihr = ihr > 0.f ? d_inter * iw : 0.f;
    const float d_ewr = ewr > 0.f ? d_area * eh : 0.f;
    const float d_ehr = ehr > 0.f ? d_area * ew : 0.f;
    float d_a0 = 0.f, d_a1 = 0.f, d_a2 = 0.f, d_a3 = 0.f;
    // intersection: rb = min(a2, b2), lt = max(a0, b0)
    if (a2 < b.x1) d_a2 += d_iwr;
    if (a0 > b.x0) d_a0 -= d_iwr;
    if (a3 < b.y1) d_a3 += d_ihr;
    if (a1 > b.y0) d_a1 -= d_ihr;
    // enclosing box: erb = max(a2, b2), elt = min(a0, b0)
    if (a2 > b.x1) d_a2 += d_ewr;
    if (a0 < b.x0) d_a0 -= d_ewr;
    if (a3 > b.y1) d_a3 += d_ehr;
    if (a1 < b.y0) d_a1 -= d_ehr;
    // area1 = (a2 - a0)(a3 - a1)
    d_a2 += d_area1 * (a3 - a1);
    d_a0 -= d_area1 * (a3 - a1);
    d_a3 += d_area1 * (a2 - a0);
    d_a1 -= d_area1 * (a2 - a0);
    grad[0] = d_a0 + d_a2;
    grad[1] = d_a1 + d_a3;
    grad[2] = s[2] > 0.f ? 0.5f * (d_a2 - d_a0) : 0.f;
    grad[3] = s[3] > 0.f ? 0.5f * (d_a3 - d_a1) : 0.f;
}

__global__ void __launch_bounds__(kLossThreads, 4)
set_loss_kernel(const float *__restrict__ logits, const float *__restrict__ boxes, const int32_t *__restrict__ labels,
                const float *__restrict__ tboxes, const int32_t *__restrict__ rows, const int32_t *__restrict__ cols,
                const uint8_t *__restrict__ valid, const float *__restrict__ num_boxes, int B, int Q, int C, int T,
                int S, float alpha, int ia_bce, float *__restrict__ losses, float *__restrict__ grad_logits,
                float *__restrict__ grad_l1, float *__restrict__ grad_giou) {
    __shared__ float red[3][kLossThreads / 32];
    const int b = blockIdx.y;
    const size_t layer = blockIdx.z;
    const int q0 = blockIdx.x * kLossRows;
    const int nrow = min(kLossRows, Q - q0);
    const float inv = 1.f / __ldg(num_boxes);
    const float a1 = (ia_bce || alpha < 0.f) ? 1.f : alpha;
    const float a0 = (ia_bce || alpha < 0.f) ? 1.f : 1.f - alpha;
    const size_t img = layer * B + b;  // (layer, image) index
    boxes += img * Q * 4;
    grad_l1 += img * Q * 4;
    grad_giou += img * Q * 4;
    rows += img * S;
    cols += img * S;
    valid += img * S;
    labels += (size_t)b * T;
    tboxes += (size_t)b * T * 4;
    losses += layer * 3;
    const size_t base = (img * Q + q0) * C;
    const float *x_tile = logits + base;
    float *g_tile = grad_logits + base;
    const int n = nrow * C;

    // Box gradients of the tile's queries: zero unless matched (overwritten below).
    for (int i = threadIdx.x; i < nrow; i += kLossThreads) {
        reinterpret_cast<float4 *>(grad_l1)[q0 + i] = make_float4(0.f, 0.f, 0.f, 0.f);
        reinterpret_cast<float4 *>(grad_giou)[q0 + i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // Dense pass: every entry as unmatched.
    float part_ce = 0.f, part_l1 = 0.f, part_giou = 0.f;
    if ((((reinterpret_cast<uintptr_t>(x_tile) | reinterpret_cast<uintptr_t>(g_tile)) & 15) | (n & 3)) == 0) {
        const int nv = n >> 2;
        const float4 *xv = reinterpret_cast<const float4 *>(x_tile);
        float4 *gv = reinterpret_cast<float4 *>(g_tile);
        for (int v0 = threadIdx.x; v0 < nv; v0 += kLossVecs * kLossThreads) {
            float4 xs[kLossVecs];
#pragma unroll
            for (int k = 0; k < kLossVecs; ++k) {
                const int v = v0 + k * kLossThreads;
                xs[k] = v < nv ? __ldcs(xv + v) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < kLossVecs; ++k) {
                const int v = v0 + k * kLossThreads;
                if (v < nv) {
                    const float2 t0 = unmatched_term(xs[k].x, a0), t1 = unmatched_term(xs[k].y, a0);
                    const float2 t2 = unmatched_term(xs[k].z, a0), t3 = unmatched_term(xs[k].w, a0);
                    part_ce += (t0.x + t1.x) + (t2.x + t3.x);
                    __stcs(gv + v, make_float4(t0.y * inv, t1.y * inv, t2.y * inv, t3.y * inv));
                }
            }
        }
    } else {
        for (int e = threadIdx.x; e < n; e += kLossThreads) {
            const float2 t = unmatched_term(__ldcs(x_tile + e), a0);
            part_ce += t.x;
            g_tile[e] = t.y * inv;
        }
    }
    __syncthreads();

    // Matched queries of the tile: box terms, and the classification entry's correction.
    // A thread reads kSlotUnroll slots' flags and rows at once, then visits its hits.
    for (int s0 = threadIdx.x; s0 < S; s0 += kSlotUnroll * kLossThreads) {
        int qs[kSlotUnroll];
        unsigned hits = 0;
#pragma unroll
        for (int k = 0; k < kSlotUnroll; ++k) {
            const int sl = s0 + k * kLossThreads;
            const bool in = sl < S;
            const int on = in ? __ldg(valid + sl) : 0;
            qs[k] = in ? __ldg(rows + sl) : -1;
            if (on && qs[k] >= q0 && qs[k] < q0 + nrow) hits |= 1u << k;
        }
        while (hits) {
            const int k = __ffs(hits) - 1;
            hits &= hits - 1;
            int q = qs[0];
#pragma unroll
            for (int kk = 1; kk < kSlotUnroll; ++kk)
                if (k == kk) q = qs[kk];
            const int sl = s0 + k * kLossThreads;
            const int t = __ldg(cols + sl);
            const int label = __ldg(labels + t);
            float sb[4], tb[4];
            const float4 s4 = __ldg(reinterpret_cast<const float4 *>(boxes) + q);
            const float4 t4 = __ldg(reinterpret_cast<const float4 *>(tboxes) + t);
            sb[0] = s4.x, sb[1] = s4.y, sb[2] = s4.z, sb[3] = s4.w;
            tb[0] = t4.x, tb[1] = t4.y, tb[2] = t4.z, tb[3] = t4.w;
            // Box losses (criterion.py:246-249).
            float4 gl;
            const float d0 = sb[0] - tb[0], d1 = sb[1] - tb[1], d2 = sb[2] - tb[2], d3 = sb[3] - tb[3];
            part_l1 += (fabsf(d0) + fabsf(d1)) + (fabsf(d2) + fabsf(d3));
            gl.x = d0 > 0.f ? inv : (d0 < 0.f ? -inv : 0.f);
            gl.y = d1 > 0.f ? inv : (d1 < 0.f ? -inv : 0.f);
            gl.z = d2 > 0.f ? inv : (d2 < 0.f ? -inv : 0.f);
            gl.w = d3 > 0.f ? inv : (d3 < 0.f ? -inv : 0.f);
            reinterpret_cast<float4 *>(grad_l1)[q] = gl;
            float lg, gg[4];
            giou_loss_grad(sb, tb, inv, lg, gg);
            part_giou += lg;
            reinterpret_cast<float4 *>(grad_giou)[q] = make_float4(gg[0], gg[1], gg[2], gg[3]);
            // Classification: replace the unmatched term of (q, label) by the matched one.
            if (label < 0 || label >= C) continue;  // next hit
            const int e = (q - q0) * C + label;
            const float x = __ldg(x_tile + e);
            float w = 0.f;
            if (ia_bce) {  // IA-BCE weight (criterion.py:189-199), stop-gradient
                const float pm = logistic(x).p;
                const float iou = iou_of(to_xyxy(sb), to_xyxy(tb));
                w = fmaxf(powf(pm, alpha) * powf(iou, 1.f - alpha), 0.01f);
            }
            const float2 m = matched_term(x, ia_bce, w, a1);
            const float2 u = unmatched_term(x, a0);
            part_ce += m.x - u.x;
            g_tile[e] = m.y * inv;
        }
    }

    // CTA sums -> global.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        part_ce += __shfl_xor_sync(0xffffffffu, part_ce, o);
        part_l1 += __shfl_xor_sync(0xffffffffu, part_l1, o);
        part_giou += __shfl_xor_sync(0xffffffffu, part_giou, o);
    }
    if (lane == 0) {
        red[0][warp] = part_ce;
        red[1][warp] = part_l1;
        red[2][warp] = part_giou;
    }
    __syncthreads();
    if (threadIdx.x < 3) {
        float sum = 0.f;
        for (int w = 0; w < kLossThreads / 32; ++w) sum += red[threadIdx.x][w];
        atomicAdd(losses + threadIdx.x, sum * inv);
    }
}

}  // namespace
}  // namespace rfdetr

using namespace rfdetr;

extern "C" int rfdetr_set_losses(void *stream, const float *pred_logits, const float *pred_boxes,
                                 const int32_t *target_labels, const float *target_boxes, const int32_t *rows,
                                 const int32_t *cols, const uint8_t *valid, const float *num_boxes, int64_t layers,
                                 int64_t batch, int64_t queries, int64_t classes, int64_t targets, int64_t slots,
                                 float focal_alpha, int32_t ia_bce, float *losses_out, float *grad_logits,
                                 float *grad_boxes_l1, float *grad_boxes_giou) {
    if (layers < 0 || batch < 0 || queries <= 0 || classes <= 0 || targets <= 0 || slots < 0 || layers > 65535 ||
        batch > 65535 || queries * classes > (1LL << 31) || layers * batch * slots > (1LL << 40))
        return RFDETR_ERR_SHAPE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (layers == 0) return RFDETR_OK;
    if (!losses_out) return RFDETR_ERR_SHAPE;
    if (cudaMemsetAsync(losses_out, 0, 3 * sizeof(float) * layers, s) != cudaSuccess) return RFDETR_ERR_CUDA;
    if (batch == 0) return RFDETR_OK;
    if (!pred_logits || !pred_boxes || !target_labels || !target_boxes || !num_boxes || !grad_logits ||
        !grad_boxes_l1 || !grad_boxes_giou || (slots > 0 && (!rows || !cols || !valid)))
        return RFDETR_ERR_SHAPE;
    // Box rows are read and written as float4.
    if ((reinterpret_cast<uintptr_t>(pred_boxes) | reinterpret_cast<uintptr_t>(target_boxes) |
         reinterpret_cast<uintptr_t>(grad_boxes_l1) | reinterpret_cast<uintptr_t>(grad_boxes_giou)) & 15)
        return RFDETR_ERR_ALIGN;
    dim3 grid((unsigned)((queries + kLossRows - 1) / kLossRows), (unsigned)batch, (unsigned)layers);
    set_loss_kernel<<<grid, kLossThreads, 0, s>>>(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols,
                                                  valid, num_boxes, (int)batch, (int)queries, (int)classes,
                                                  (int)targets, (int)slots, focal_alpha, ia_bce != 0, losses_out,
                                                  grad_logits, grad_boxes_l1, grad_boxes_giou);
    return launch_status();
}
