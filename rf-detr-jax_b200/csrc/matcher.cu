// Matching cost and batched exact assignment for sm_100a.
//
// Cost: build_cost_matrix for classes and boxes (src/rfdetr_jax/models/matcher.py:44-103,141;
// focal term :36-41; GIoU src/rfdetr_jax/utilities/box_ops.py:27-75).
//
// Assignment: hungarian_match / _solve_batch (matcher.py:144-208), which calls
// scipy.optimize.linear_sum_assignment per (image, group) block.  SciPy solves with Crouse's
// shortest augmenting path (IEEE TAES 52(4), 2016) in float64; this kernel runs the same method
// with the same tie rules, so its answer is SciPy's bit for bit:
//   * a tall block (more queries than targets, the usual case) is solved transposed and reported
//     in ascending query order;
//   * rows are inserted in index order; each insertion scans the unscanned columns through a
//     work list that starts in descending column order and drops a column by moving the list's
//     last entry into its slot;
//   * reduced cost ((minVal + c) - u[i]) - v[j]; the next column has the smallest tentative
//     distance, ties going to an unassigned column (the later one in the work list), else to the
//     earliest one in the work list.
// One CTA solves one block: the column scan of each augmenting step is spread over the CTA's
// threads and the arg-min is a CTA reduction under that tie order.  Blocks of up to 384 columns
// run lsap_reg_kernel (each column's state in its thread's registers; its leading rows staged in
// shared memory up to the largest per-CTA budget that keeps two CTAs on an SM, the rest read
// through L1); wider blocks run lsap_list_kernel (state and work list in shared memory, the block
// staged when it fits that budget).
#include <algorithm>

#include "common.cuh"

namespace rfdetr {
namespace {

// ------------------------------------------------------------------------------------------
// Cost
// ------------------------------------------------------------------------------------------
constexpr int kCostThreads = 256;
constexpr int kTargetFields = 10;  // label, mask, cx, cy, w, h, x0, y0, x1, y1

template <typename T> __device__ __forceinline__ float ldf(const T *p) { return to_f32(__ldg(p)); }

template <typename TL, typename TB>
__global__ void __launch_bounds__(kCostThreads)
match_cost_kernel(const TL *__restrict__ logits, const TB *__restrict__ boxes, const int32_t *__restrict__ labels,
                  const float *__restrict__ tboxes, const uint8_t *__restrict__ tmask, float *__restrict__ cost,
                  int Q, int C, int T, int q_tile, int target_batch, float cost_class, float cost_bbox,
                  float cost_giou, float alpha) {
    extern __shared__ float tsm[];  // [kTargetFields][T]
    const int b = blockIdx.y;                 // (layer, image) row of the predictions and the cost
    const int bt = blockIdx.y % target_batch;  // image of the targets (shared by stacked layers)
    const int q0 = blockIdx.x * q_tile;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float cx = __ldg(tboxes + ((size_t)bt * T + t) * 4 + 0);
        const float cy = __ldg(tboxes + ((size_t)bt * T + t) * 4 + 1);
        const float w = __ldg(tboxes + ((size_t)bt * T + t) * 4 + 2);
        const float h = __ldg(tboxes + ((size_t)bt * T + t) * 4 + 3);
        const float wc = fmaxf(w, 0.f), hc = fmaxf(h, 0.f);  // box_ops.py:30-31 clip
        tsm[0 * T + t] = __int_as_float(__ldg(labels + (size_t)bt * T + t));
        tsm[1 * T + t] = __ldg(tmask + (size_t)bt * T + t) ? 1.f : 0.f;
        tsm[2 * T + t] = cx;
        tsm[3 * T + t] = cy;
        tsm[4 * T + t] = w;
        tsm[5 * T + t] = h;
        tsm[6 * T + t] = cx - 0.5f * wc;
        tsm[7 * T + t] = cy - 0.5f * hc;
        tsm[8 * T + t] = cx + 0.5f * wc;
        tsm[9 * T + t] = cy + 0.5f * hc;
    }
    __syncthreads();
    // One warp per query row: the prediction's box terms are computed once per lane, lanes walk
    // the targets (consecutive lanes, consecutive targets: coalesced stores).  Divisions, exp and
    // log use the fast hardware forms; their errors (a few ulp, about 1e-7 relative) sit far
    // inside the float32 cost tolerance.
    const int q1 = min(q0 + q_tile, Q);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const float qnan = __int_as_float(0x7fc00000);
    for (int q = q0 + warp; q < q1; q += nwarps) {
        const size_t qrow = (size_t)b * Q + q;
        const float pcx = ldf(boxes + qrow * 4 + 0), pcy = ldf(boxes + qrow * 4 + 1);
        const float pw = ldf(boxes + qrow * 4 + 2), ph = ldf(boxes + qrow * 4 + 3);
        const float pwc = fmaxf(pw, 0.f), phc = fmaxf(ph, 0.f);  // box_ops.py:30-31 clip
        const float ax0 = pcx - 0.5f * pwc, ay0 = pcy - 0.5f * phc;
        const float ax1 = pcx + 0.5f * pwc, ay1 = pcy + 0.5f * phc;
        const float area1 = (ax1 - ax0) * (ay1 - ay0);
        const TL *lrow = logits + qrow * C;
        // The reference reads a target's logit through a one-hot contraction (matcher.py:92-93):
        // a non-finite logit at any other class contributes x * 0 = NaN to every target of the
        // row.  Count the row's non-finite logits once.
        int nbad = 0;
        for (int c = lane; c < C; c += 32) nbad += isfinite(ldf(lrow + c)) ? 0 : 1;
        nbad = __reduce_add_sync(0xffffffffu, nbad);
        for (int t = lane; t < T; t += 32) {
            float out;
            if (tsm[1 * T + t] == 0.f) {
                out = 1e4f;  // matcher.py:141
            } else {
                const int label = __float_as_int(tsm[0 * T + t]);
                // Focal classification cost (matcher.py:36-41) on the target's own logit.
                // A label outside [0, C) has an all-zero one-hot row: its logit reads as 0.
                float x = 0.f;
                if (label >= 0 && label < C) x = ldf(lrow + label);
                if (nbad - (isfinite(x) ? 0 : 1) > 0 || x != x) x = qnan;
                float cls;
                {
                    const float e_ = __expf(-fabsf(x));
                    const float u = 1.f + e_;
                    const float l1p = __logf(u);                // log1p(e): u - 1 >= 0.0067 unless e_ is tiny
                    const float sp_pos = fmaxf(x, 0.f) + l1p;   // -log_sigmoid(-x)
                    const float sp_neg = fmaxf(-x, 0.f) + l1p;  // -log_sigmoid(x)
                    const float inv = __fdividef(1.f, u);
                    const float p = x >= 0.f ? inv : e_ * inv;   // sigmoid(x)
                    const float pm = x >= 0.f ? e_ * inv : inv;  // 1 - sigmoid(x)
                    const float negative = (1.f - alpha) * (p * p) * sp_pos;
                    const float positive = alpha * (pm * pm) * sp_neg;
                    cls = x != x ? qnan : positive - negative;
                }
                const float l1 = ((fabsf(pcx - tsm[2 * T + t]) + fabsf(pcy - tsm[3 * T + t])) +
                                  fabsf(pw - tsm[4 * T + t])) + fabsf(ph - tsm[5 * T + t]);
                // GIoU (box_ops.py:46-75) on xyxy boxes.
                const float bx0 = tsm[6 * T + t], by0 = tsm[7 * T + t];
                const float bx1 = tsm[8 * T + t], by1 = tsm[9 * T + t];
                const float area2 = (bx1 - bx0) * (by1 - by0);
                const float iw = fmaxf(fminf(ax1, bx1) - fmaxf(ax0, bx0), 0.f);
                const float ih = fmaxf(fminf(ay1, by1) - fmaxf(ay0, by0), 0.f);
                const float inter = iw * ih;
                const float uni = area1 + area2 - inter;
                const float iou = __fdividef(inter, fmaxf(uni, 1e-7f));
                const float ew = fmaxf(fmaxf(ax1, bx1) - fminf(ax0, bx0), 0.f);
                const float eh = fmaxf(fmaxf(ay1, by1) - fminf(ay0, by0), 0.f);
                const float area = ew * eh;
                const float giou = iou - __fdividef(area - uni, fmaxf(area, 1e-7f));
                out = cost_bbox * l1 + cost_class * cls + cost_giou * (-giou);
            }
            cost[qrow * T + t] = out;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Assignment
// ------------------------------------------------------------------------------------------
constexpr int kLsapThreads = 128;
constexpr int kLsapWarps = kLsapThreads / 32;
constexpr int kLsapMaxTargets = 1024;
constexpr int kLsapMaxGroup = 4096;
constexpr int kScanUnroll = 3;  // columns per thread per pass of a scan step (300 columns / 128 threads)

struct Cand {
    double d;
    int k;     // position in the work list, -1 = none
    int free;  // column unassigned
};

// True if a beats b under SciPy's selection order (see file comment).
__device__ __forceinline__ bool beats(const Cand &a, const Cand &b) {
    if (a.k < 0) return false;
    if (b.k < 0) return true;
    if (a.d < b.d) return true;
    if (a.d > b.d) return false;
    if (a.free != b.free) return a.free != 0;
    return a.free ? (a.k > b.k) : (a.k < b.k);
}

__device__ __forceinline__ Cand shfl_cand(const Cand &c, int o) {
    Cand r;
    r.d = __shfl_xor_sync(0xffffffffu, c.d, o);
    r.k = __shfl_xor_sync(0xffffffffu, c.k, o);
    r.free = __shfl_xor_sync(0xffffffffu, c.free, o);
    return r;
}

struct LsapArgs {
    const float *cost;
    const int32_t *sizes;  // problem n (a (layer, image) row of the cost) uses sizes[n % size_mod]
    int size_mod;
    int Q, T, G, Qg;
    int smem_cost_floats;  // capacity of the shared cost stage (0 = never stage)
    int step_cap;          // scan steps an augmenting path may take before the solve gives up
    int32_t *rows, *cols;
    uint8_t *valid;
    int32_t *status;
};

// Writes a solved block's assignment: a wide or square block by row; a transposed one with the
// assigned queries in ascending order (a block-wide compaction).
__device__ void report_assignment(const LsapArgs &a, size_t obase, int start, bool tr, int nr, int nc,
                                  const int *col4row, const int *row4col) {
    const int tid = threadIdx.x;
    if (!tr) {
        for (int i = tid; i < nr; i += kLsapThreads) {
            a.rows[obase + i] = start + i;
            a.cols[obase + i] = col4row[i];
            a.valid[obase + i] = 1;
        }
        return;
    }
    __shared__ int s_warp_count[kLsapWarps];
    __shared__ int s_base;
    if (tid == 0) s_base = 0;
    __syncthreads();
    for (int j0 = 0; j0 < nc; j0 += kLsapThreads) {
        const int j = j0 + tid;
        const bool on = j < nc && row4col[j] >= 0;
        const unsigned bal = __ballot_sync(0xffffffffu, on);
        const int lane = tid & 31, w = tid >> 5;
        if (lane == 0) s_warp_count[w] = __popc(bal);
        __syncthreads();
        int before = s_base;
        for (int k = 0; k < w; ++k) before += s_warp_count[k];
        if (on) {
            const int slot = before + __popc(bal & ((1u << lane) - 1u));
            a.rows[obase + slot] = start + j;
            a.cols[obase + slot] = row4col[j];
            a.valid[obase + slot] = 1;
        }
        __syncthreads();
        if (tid == 0) {
            int total = 0;
            for (int k = 0; k < kLsapWarps; ++k) total += s_warp_count[k];
            s_base += total;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kLsapThreads) lsap_list_kernel(const LsapArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int tid = threadIdx.x;
    const int prob = blockIdx.x;
    const int n = prob / a.G, g = prob - (prob / a.G) * a.G;
    const int Qg = a.Qg, T = a.T;
    const int start = g * Qg;
    const size_t obase = ((size_t)n * a.G + g) * T;
    for (int k = tid; k < T; k += kLsapThreads) {
        a.rows[obase + k] = 0;
        a.cols[obase + k] = 0;
        a.valid[obase + k] = 0;
    }
    int size = __ldg(a.sizes + n % a.size_mod);
    size = max(0, min(size, T));
    if (size == 0) return;

    const bool tr = size < Qg;  // solve transposed: rows = targets, columns = queries
    const int nr = tr ? size : Qg;
    const int nc = tr ? Qg : size;
    const int M = max(Qg, T);

    double *u = reinterpret_cast<double *>(sm);
    double *v = u + M;
    double *dist = v + M;
    int *path = reinterpret_cast<int *>(dist + M);
    int *col4row = path + M;
    int *row4col = col4row + M;
    int *todo = row4col + M;
    unsigned char *rseen = reinterpret_cast<unsigned char *>(todo + M);
    unsigned char *cseen = rseen + M;
    Cand *red = reinterpret_cast<Cand *>(cseen + ((2 * M + 15) & ~15) - M);
    __shared__ int s_i, s_sink, s_left, s_fail;
    __shared__ double s_minv;
    __shared__ float s_sentinel;
    float *csm = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(red) + kLsapWarps * sizeof(Cand) + 16);
    csm = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(csm) + 15) & ~(uintptr_t)15);

    // Stage the block (queries x real targets), find non-finite entries and the finite max.
    const float *gblock = a.cost + ((size_t)n * a.Q + start) * T;
    const bool staged = (long long)Qg * size <= (long long)a.smem_cost_floats;
    float fmax_local = -INFINITY;
    int bad_local = 0;
    for (int e = tid; e < Qg * size; e += kLsapThreads) {
        const int qi = e / size, ti = e - (e / size) * size;
        const float c = __ldg(gblock + (size_t)qi * T + ti);
        if (staged) csm[e] = c;
        if (isfinite(c)) fmax_local = fmaxf(fmax_local, c);
        else bad_local = 1;
    }
    const int any_bad = __syncthreads_or(bad_local);
    float sentinel = 0.f;
    if (any_bad) {
        // matcher.py:169-172: non-finite entries become max(finite) + 1 (float32), or 1.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) fmax_local = fmaxf(fmax_local, __shfl_xor_sync(0xffffffffu, fmax_local, o));
        __shared__ float s_wmax[kLsapWarps];
        if ((tid & 31) == 0) s_wmax[tid >> 5] = fmax_local;
        __syncthreads();
        if (tid == 0) {
            float m = -INFINITY;
            for (int w = 0; w < kLsapWarps; ++w) m = fmaxf(m, s_wmax[w]);
            s_sentinel = (m == -INFINITY) ? 1.f : __fadd_rn(m, 1.f);
        }
        __syncthreads();
        sentinel = s_sentinel;
        if (staged) {
            for (int e = tid; e < Qg * size; e += kLsapThreads)
                if (!isfinite(csm[e])) csm[e] = sentinel;
        }
    }
    // Solver-orientation cost C(i, j) as float64.
    auto cost_at = [&](int i, int j) -> double {
        const int qi = tr ? j : i, ti = tr ? i : j;
        float c;
        if (staged) {
            c = csm[qi * size + ti];
        } else {
            c = __ldg(gblock + (size_t)qi * T + ti);
            if (any_bad && !isfinite(c)) c = sentinel;
        }
        return (double)c;
    };

    for (int j = tid; j < nc; j += kLsapThreads) {
        v[j] = 0.0;
        row4col[j] = -1;
        path[j] = -1;
    }
    for (int i = tid; i < nr; i += kLsapThreads) {
        u[i] = 0.0;
        col4row[i] = -1;
    }
    if (tid == 0) s_fail = 0;
    __syncthreads();

    for (int cur = 0; cur < nr; ++cur) {
        for (int j = tid; j < nc; j += kLsapThreads) {
            dist[j] = INFINITY;
            cseen[j] = 0;
            todo[j] = nc - 1 - j;
        }
        for (int i = tid; i < nr; i += kLsapThreads) rseen[i] = 0;
        if (tid == 0) {
            s_i = cur;
            s_sink = -1;
            s_left = nc;
            s_minv = 0.0;
        }
        __syncthreads();

        const int steps = min(nc, a.step_cap - 1);
        for (int step = 0; step <= steps; ++step) {  // each step retires one column
            const int i = s_i;
            const int left = s_left;
            const double minv = s_minv;
            if (tid == 0) rseen[i] = 1;
            const double ui = u[i];
            Cand best;
            best.d = INFINITY;
            best.k = -1;
            best.free = 0;
            // kScanUnroll of the thread's columns at a time, all their loads issued before the
            // arithmetic (the work-list entry, then the column's cost, v, dist and owner).
            for (int k0 = tid; k0 < left; k0 += kScanUnroll * kLsapThreads) {
                int jj[kScanUnroll];
#pragma unroll
                for (int u = 0; u < kScanUnroll; ++u) {
                    const int k = k0 + u * kLsapThreads;
                    jj[u] = k < left ? todo[k] : -1;
                }
                float cc[kScanUnroll];
                double vv[kScanUnroll], dd[kScanUnroll];
                int owner[kScanUnroll];
#pragma unroll
                for (int u = 0; u < kScanUnroll; ++u) {
                    const int j = jj[u];
                    if (j >= 0) {
                        cc[u] = (float)cost_at(i, j);
                        vv[u] = v[j];
                        dd[u] = dist[j];
                        owner[u] = row4col[j];
                    }
                }
#pragma unroll
                for (int u = 0; u < kScanUnroll; ++u) {
                    const int j = jj[u];
                    if (j < 0) continue;
                    const double r = __dsub_rn(__dsub_rn(__dadd_rn(minv, (double)cc[u]), ui), vv[u]);
                    double d = dd[u];
                    if (r < d) {
                        path[j] = i;
                        dist[j] = r;
                        d = r;
                    }
                    Cand c;
                    c.d = d;
                    c.k = k0 + u * kLsapThreads;
                    c.free = owner[u] == -1;
                    if (beats(c, best)) best = c;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const Cand other = shfl_cand(best, o);
                if (beats(other, best)) best = other;
            }
            if ((tid & 31) == 0) red[tid >> 5] = best;
            __syncthreads();
            if (tid == 0) {
                Cand b = red[0];
                for (int w = 1; w < kLsapWarps; ++w)
                    if (beats(red[w], b)) b = red[w];
                if (b.k < 0 || b.d == INFINITY) {
                    s_fail = 1;
                } else {
                    const int j = todo[b.k];
                    if (row4col[j] == -1) s_sink = j;
                    else s_i = row4col[j];
                    cseen[j] = 1;
                    todo[b.k] = todo[left - 1];
                    s_left = left - 1;
                    s_minv = b.d;
                }
            }
            __syncthreads();
            if (s_fail || s_sink != -1) break;
        }
        if (s_sink == -1) s_fail = 1;  // the scan cap was reached (cannot happen for finite costs)
        if (s_fail) break;

        const double minv = s_minv;
        for (int r = tid; r < nr; r += kLsapThreads)
            if (rseen[r] && r != cur) u[r] = __dadd_rn(u[r], __dsub_rn(minv, dist[col4row[r]]));
        for (int c = tid; c < nc; c += kLsapThreads)
            if (cseen[c]) v[c] = __dsub_rn(v[c], __dsub_rn(minv, dist[c]));
        __syncthreads();  // the dual update reads col4row, which the path walk rewrites
        if (tid == 0) {
            u[cur] = __dadd_rn(u[cur], minv);
            int j = s_sink;
            for (int hop = 0; hop <= nr; ++hop) {
                const int r = path[j];
                row4col[j] = r;
                const int t = col4row[r];
                col4row[r] = j;
                j = t;
                if (r == cur) break;
                if (hop == nr) s_fail = 1;
            }
        }
        __syncthreads();
        if (s_fail) break;
    }

    if (s_fail) {
        if (tid == 0) atomicExch(a.status, (int)RFDETR_ERR_LIMIT);
        return;
    }
    report_assignment(a, obase, start, tr, nr, nc, col4row, row4col);
}

// Order-preserving 64-bit key of a float64 distance (+0 and -0 share one key, as they compare
// equal), and its inverse.
__device__ __forceinline__ unsigned long long dist_key(double d) {
    const unsigned long long bits = (unsigned long long)__double_as_longlong(d + 0.0);
    return bits ^ ((bits >> 63) ? 0xffffffffffffffffull : 0x8000000000000000ull);
}
__device__ __forceinline__ double dist_of_key(unsigned long long key) {
    key ^= (key >> 63) ? 0x8000000000000000ull : 0xffffffffffffffffull;
    return __longlong_as_double((long long)key);
}

// Tie key of a column at work-list position `pos`: smaller wins; unassigned columns first, the
// later one among them, else the earliest (the order of `beats`).
__device__ __forceinline__ unsigned tie_key(bool free, int pos) {
    return free ? (0xffffu - (unsigned)pos) : (0x10000u | (unsigned)pos);
}

// The solver for blocks of up to R * 128 columns: the same method, tie rules and float64
// arithmetic as lsap_list_kernel, with each column owned by a fixed thread (column c by thread
// c % 128) that keeps the column's dual, tentative distance, owner row and work-list position in
// registers.  The work list exists only as those positions (SciPy's swap-remove moves the list's
// last column into the retired column's slot, so each step updates one position), which keeps
// the tie order exact.  A scan step then reads from shared memory only the row's dual and its
// costs: its candidate is the minimum of a 96-bit key (distance, tie key) over the CTA -- three
// redux.sync minimums per warp, then every thread combines the four warp minimums itself, and
// the winning column's owner publishes the next row.  The dual update runs from the column side
// (a row seen by the search, other than the inserted one, owns exactly one retired column) before
// the path is flipped.
template <int R>
__global__ void __launch_bounds__(kLsapThreads, 2) lsap_reg_kernel(const LsapArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int tid = threadIdx.x;
    const int prob = blockIdx.x;
    const int n = prob / a.G, g = prob - (prob / a.G) * a.G;
    const int Qg = a.Qg, T = a.T;
    const int start = g * Qg;
    const size_t obase = ((size_t)n * a.G + g) * T;
    for (int k = tid; k < T; k += kLsapThreads) {
        a.rows[obase + k] = 0;
        a.cols[obase + k] = 0;
        a.valid[obase + k] = 0;
    }
    int size = __ldg(a.sizes + n % a.size_mod);
    size = max(0, min(size, T));
    if (size == 0) return;

    const bool tr = size < Qg;  // solve transposed: rows = targets, columns = queries
    const int nr = tr ? size : Qg;
    const int nc = tr ? Qg : size;
    const int M = max(Qg, T);

    double *u = reinterpret_cast<double *>(sm);
    int *path = reinterpret_cast<int *>(u + M);
    int *col4row = path + M;
    int *row4col = col4row + M;
    float *csm = reinterpret_cast<float *>(row4col + M);
    csm = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(csm) + 15) & ~(uintptr_t)15);
    __shared__ int s_bad;
    __shared__ float s_sentinel;
    __shared__ unsigned s_red[2][kLsapWarps][3];  // by step parity: one barrier per step

    // Stage the block's first rows (solver orientation) row-major, so a step reads consecutive
    // columns; rows past the stage are read from global memory.  Also find non-finite entries
    // and the finite max.
    const float *gblock = a.cost + ((size_t)n * a.Q + start) * T;
    const int srows = min(nr, a.smem_cost_floats / nc);
    float fmax_local = -INFINITY;
    int bad_local = 0;
    for (int e = tid; e < Qg * size; e += kLsapThreads) {
        const int qi = e / size, ti = e - (e / size) * size;
        const float c = __ldg(gblock + (size_t)qi * T + ti);
        const int i = tr ? ti : qi, j = tr ? qi : ti;
        if (i < srows) csm[i * nc + j] = c;
        if (isfinite(c)) fmax_local = fmaxf(fmax_local, c);
        else bad_local = 1;
    }
    const int any_bad = __syncthreads_or(bad_local);
    float sentinel = 0.f;
    if (any_bad) {
        // matcher.py:169-172: non-finite entries become max(finite) + 1 (float32), or 1.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) fmax_local = fmaxf(fmax_local, __shfl_xor_sync(0xffffffffu, fmax_local, o));
        __shared__ float s_wmax[kLsapWarps];
        if ((tid & 31) == 0) s_wmax[tid >> 5] = fmax_local;
        __syncthreads();
        if (tid == 0) {
            float m = -INFINITY;
            for (int w = 0; w < kLsapWarps; ++w) m = fmaxf(m, s_wmax[w]);
            s_sentinel = (m == -INFINITY) ? 1.f : __fadd_rn(m, 1.f);
        }
        __syncthreads();
        sentinel = s_sentinel;
        for (int e = tid; e < srows * nc; e += kLsapThreads)
            if (!isfinite(csm[e])) csm[e] = sentinel;
    }
    const int gstride = tr ? T : 1;

    // Column state, column c = tid + q * kLsapThreads.
    double cv[R], cd[R];
    int cpos[R], cown[R];
    unsigned live = 0, seen = 0;  // bit q: column in the work list / retired in this insertion
#pragma unroll
    for (int q = 0; q < R; ++q) {
        const int c = tid + q * kLsapThreads;
        cv[q] = 0.0;
        cd[q] = INFINITY;
        cpos[q] = nc - 1 - c;  // the work list starts in descending column order
        cown[q] = -1;
        if (c < nc) live |= 1u << q;
    }
    const unsigned all_live = live;
    for (int r = tid; r < M; r += kLsapThreads) {
        u[r] = 0.0;
        col4row[r] = -1;
        row4col[r] = -1;
    }
    if (tid == 0) s_bad = 0;
    __syncthreads();

    bool fail = false;
    const int steps = min(nc, a.step_cap - 1);
    for (int cur = 0; cur < nr && !fail; ++cur) {
        int i = cur, left = nc, sink = -1;
        double minv = 0.0;
        for (int step = 0; step <= steps; ++step) {  // each step retires one column
            const double ui = u[i];
            const float *srow = i < srows ? csm + i * nc : nullptr;
            const float *grow = tr ? gblock + i : gblock + (size_t)i * T;
            unsigned long long bkey = ~0ull;
            unsigned btie = 0xffffffffu;
#pragma unroll
            for (int q = 0; q < R; ++q) {
                if (!((live >> q) & 1u)) continue;
                const int c = tid + q * kLsapThreads;
                float cc;
                if (srow) {
                    cc = srow[c];
                } else {
                    cc = __ldg(grow + (size_t)c * gstride);
                    if (any_bad && !isfinite(cc)) cc = sentinel;
                }
                const double r = __dsub_rn(__dsub_rn(__dadd_rn(minv, (double)cc), ui), cv[q]);
                if (r < cd[q]) {
                    cd[q] = r;
                    path[c] = i;
                }
                const unsigned long long key = dist_key(cd[q]);
                const unsigned tk = (tie_key(cown[q] == -1, cpos[q]) << 9) | (unsigned)c;
                if (key < bkey || (key == bkey && tk < btie)) {
                    bkey = key;
                    btie = tk;
                }
            }
            const unsigned w1 = (unsigned)(bkey >> 32), w2 = (unsigned)bkey;
            const unsigned m1 = __reduce_min_sync(0xffffffffu, w1);
            const bool e1 = w1 == m1;
            const unsigned m2 = __reduce_min_sync(0xffffffffu, e1 ? w2 : 0xffffffffu);
            const bool e2 = e1 && w2 == m2;
            const unsigned m3 = __reduce_min_sync(0xffffffffu, e2 ? btie : 0xffffffffu);
            unsigned(*red)[3] = s_red[step & 1];
            if ((tid & 31) == 0) {
                red[tid >> 5][0] = m1;
                red[tid >> 5][1] = m2;
                red[tid >> 5][2] = m3;
            }
            __syncthreads();
            unsigned b1 = red[0][0], b2 = red[0][1], b3 = red[0][2];
#pragma unroll
            for (int w = 1; w < kLsapWarps; ++w) {
                const unsigned x1 = red[w][0], x2 = red[w][1], x3 = red[w][2];
                if (x1 < b1 || (x1 == b1 && (x2 < b2 || (x2 == b2 && x3 < b3)))) {
                    b1 = x1;
                    b2 = x2;
                    b3 = x3;
                }
            }
            const unsigned long long wkey = ((unsigned long long)b1 << 32) | b2;
            if (b3 == 0xffffffffu || wkey >= dist_key(INFINITY)) {  // no column, or none reachable
                fail = true;
                break;
            }
            // The winner: its work-list position and, in the tie word's low bits, its column --
            // whose row every thread reads from row4col (fixed during the scan).
            const unsigned wt = b3 >> 9;
            const int kwin = (wt & 0x10000u) ? (int)(wt & 0xffffu) : (int)(0xffffu - wt);
            const int cwin = (int)(b3 & 511u);
            // The winning column leaves the list; the column in the list's last slot takes its
            // position.
#pragma unroll
            for (int q = 0; q < R; ++q) {
                if (!((live >> q) & 1u)) continue;
                if (cpos[q] == kwin) {
                    live &= ~(1u << q);
                    seen |= 1u << q;
                } else if (cpos[q] == left - 1) {
                    cpos[q] = kwin;
                }
            }
            --left;
            minv = dist_of_key(wkey);
            const int next = row4col[cwin];
            if (next == -1) {
                sink = cwin;
                break;
            }
            i = next;
        }
        if (sink == -1) fail = true;  // no reachable column, or the scan cap was reached
        if (fail) break;

        // Dual update, then the next insertion's column state; the path flips after a barrier.
#pragma unroll
        for (int q = 0; q < R; ++q) {
            if ((seen >> q) & 1u) {
                const double dm = __dsub_rn(minv, cd[q]);
                cv[q] = __dsub_rn(cv[q], dm);
                if (cown[q] >= 0) u[cown[q]] = __dadd_rn(u[cown[q]], dm);
            }
            cd[q] = INFINITY;
            cpos[q] = nc - 1 - (tid + q * kLsapThreads);
        }
        seen = 0;
        live = all_live;
        __syncthreads();
        if (tid == 0) {
            u[cur] = __dadd_rn(u[cur], minv);
            int j = sink;
            for (int hop = 0; hop <= nr; ++hop) {
                const int r = path[j];
                row4col[j] = r;
                const int t = col4row[r];
                col4row[r] = j;
                j = t;
                if (r == cur) break;
                if (hop == nr) s_bad = 1;
            }
        }
        __syncthreads();
        if (s_bad) {
            fail = true;
            break;
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int c = tid + q * kLsapThreads;
            if (c < nc) cown[q] = row4col[c];
        }
    }

    if (fail) {
        if (tid == 0) atomicExch(a.status, (int)RFDETR_ERR_LIMIT);
        return;
    }
    report_assignment(a, obase, start, tr, nr, nc, col4row, row4col);
}

// Shared-memory state of lsap_reg_kernel, before the cost stage.
size_t lsap_reg_state_bytes(int M) {
    return ((size_t)M * sizeof(double) + 3 * (size_t)M * sizeof(int) + 15 + 15) & ~(size_t)15;
}

size_t lsap_state_bytes(int M) {
    size_t b = 3 * (size_t)M * sizeof(double) + 4 * (size_t)M * sizeof(int);
    b += ((2 * (size_t)M + 15) & ~(size_t)15);
    b += kLsapWarps * sizeof(Cand) + 32;
    return (b + 15) & ~(size_t)15;
}

}  // namespace
}  // namespace rfdetr

using namespace rfdetr;

namespace {

// The cost of `batch` prediction rows (a row: Q queries), row y against target image
// y % target_batch.
int launch_match_cost(void *stream, const void *pred_logits, int logits_dtype, const void *pred_boxes,
                      int boxes_dtype, const int32_t *target_labels, const float *target_boxes,
                      const uint8_t *target_mask, float *cost, int64_t batch, int64_t target_batch, int64_t queries,
                      int64_t classes, int64_t targets, float cost_class, float cost_bbox, float cost_giou,
                      float focal_alpha) {
    if ((logits_dtype != RFDETR_F32 && logits_dtype != RFDETR_BF16) ||
        (boxes_dtype != RFDETR_F32 && boxes_dtype != RFDETR_BF16))
        return RFDETR_ERR_DTYPE;
    if (batch < 0 || queries < 0 || classes <= 0 || targets < 0 || batch > 65535 ||
        batch * queries * (classes > targets ? classes : targets) > (1LL << 31) || targets > 4096)
        return RFDETR_ERR_SHAPE;
    if (batch == 0 || queries == 0 || targets == 0) return RFDETR_OK;
    if (!pred_logits || !pred_boxes || !target_labels || !target_boxes || !target_mask || !cost)
        return RFDETR_ERR_SHAPE;
    const int ls = dtype_size(logits_dtype), bs = dtype_size(boxes_dtype);
    if (!aligned(pred_logits, ls) || !aligned(pred_boxes, bs) || !aligned(target_labels, 4) ||
        !aligned(target_boxes, 4) || !aligned(cost, 4))
        return RFDETR_ERR_ALIGN;
    const int T = (int)targets;
    const int q_tile = std::max(1, (int)std::min<long long>(queries, std::max<long long>(1, 4096 / T)));
    dim3 grid((unsigned)ceil_div(queries, q_tile), (unsigned)batch);
    const size_t smem = (size_t)kTargetFields * T * sizeof(float);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define RFDETR_COST_LAUNCH(TL, TB)                                                                        \
    match_cost_kernel<TL, TB><<<grid, kCostThreads, smem, s>>>(                                           \
        static_cast<const TL *>(pred_logits), static_cast<const TB *>(pred_boxes), target_labels,        \
        target_boxes, target_mask, cost, (int)queries, (int)classes, T, q_tile, (int)target_batch,      \
        cost_class, cost_bbox, cost_giou, focal_alpha)
    if (logits_dtype == RFDETR_F32 && boxes_dtype == RFDETR_F32) RFDETR_COST_LAUNCH(float, float);
    else if (logits_dtype == RFDETR_F32) RFDETR_COST_LAUNCH(float, bf16);
    else if (boxes_dtype == RFDETR_F32) RFDETR_COST_LAUNCH(bf16, float);
    else RFDETR_COST_LAUNCH(bf16, bf16);
#undef RFDETR_COST_LAUNCH
    return launch_status();
}

// The exact assignment of `problems` cost rows (a row: Q x T), row n with sizes[n % size_mod].
int launch_lsap(void *stream, const float *cost, const int32_t *sizes, int64_t size_mod, int64_t problems,
                int64_t queries, int64_t max_targets, int64_t group_detr, int32_t *rows, int32_t *cols,
                uint8_t *valid, int32_t *status_out) {
    if (problems < 0 || queries <= 0 || max_targets <= 0 || group_detr <= 0 || queries % group_detr != 0 ||
        max_targets > kLsapMaxTargets || queries / group_detr > kLsapMaxGroup ||
        problems * group_detr > 2147483647LL || problems * queries * max_targets > (1LL << 40))
        return RFDETR_ERR_SHAPE;
    if (problems == 0) return RFDETR_OK;
    if (!cost || !sizes || !rows || !cols || !valid || !status_out) return RFDETR_ERR_SHAPE;
    if (!aligned(cost, 4) || !aligned(sizes, 4) || !aligned(rows, 4) || !aligned(cols, 4) ||
        !aligned(status_out, 4))
        return RFDETR_ERR_ALIGN;
    LsapArgs a;
    a.cost = cost;
    a.sizes = sizes;
    a.size_mod = (int)size_mod;
    a.Q = (int)queries;
    a.T = (int)max_targets;
    a.G = (int)group_detr;
    a.Qg = (int)(queries / group_detr);
    a.rows = rows;
    a.cols = cols;
    a.valid = valid;
    a.status = status_out;
    const int M = std::max(a.Qg, a.T);
    // Blocks of up to 384 columns (the column count of a block is at most max(Qg, T)) take the
    // register-resident solver; wider ones the work-list solver.
    const int R = M <= kLsapThreads ? 1 : M <= 2 * kLsapThreads ? 2 : M <= 3 * kLsapThreads ? 3 : 0;
    const void *fn = R == 1 ? (const void *)lsap_reg_kernel<1>
                   : R == 2 ? (const void *)lsap_reg_kernel<2>
                   : R == 3 ? (const void *)lsap_reg_kernel<3>
                            : (const void *)lsap_list_kernel;
    const size_t state = R ? lsap_reg_state_bytes(M) : lsap_state_bytes(M);
    // Stage budget: the most shared memory a CTA can take while two still fit an SM.  A
    // transposed solve reads one target's cost for every query per scan step, so staging the
    // block's rows keeps the step in shared memory; two CTAs per SM (one short second wave at
    // config 4) measured faster than three with smaller stages.  The RFDETR_LSAP_STAGE_KB knob
    // overrides it.
    int dev = 0, optin = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaFuncAttributes fa{};
    const size_t static_bytes = cudaFuncGetAttributes(&fa, fn) == cudaSuccess ? fa.sharedSizeBytes : 0;
    const size_t half = (size_t)per_sm / 2;
    size_t budget = half > 1024 + static_bytes ? ((half - 1024 - static_bytes) & ~(size_t)15) : 0;
    const KnobValue stage_kb = knob(kKnobLsapStageKb);
    if (stage_kb.count > 0) budget = (size_t)std::max(stage_kb.v[0], 0) * 1024;
    const KnobValue step_cap = knob(kKnobLsapStepCap);
    a.step_cap = step_cap.count > 0 ? std::max(step_cap.v[0], 1) : 0x7fffffff;
    const size_t want = (size_t)a.Qg * a.T * sizeof(float);
    size_t stage = std::min(want, budget > state ? budget - state : 0);
    if (state + stage > (size_t)optin) stage = (size_t)optin > state ? (size_t)optin - state : 0;
    stage &= ~(size_t)15;
    a.smem_cost_floats = (int)(stage / sizeof(float));
    const size_t smem = state + stage;
    if (smem > (size_t)optin) return RFDETR_ERR_SHAPE;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return RFDETR_ERR_CUDA;
    const dim3 grid((unsigned)(problems * group_detr)), block(kLsapThreads);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (R) {
        case 1: lsap_reg_kernel<1><<<grid, block, smem, s>>>(a); break;
        case 2: lsap_reg_kernel<2><<<grid, block, smem, s>>>(a); break;
        case 3: lsap_reg_kernel<3><<<grid, block, smem, s>>>(a); break;
        default: lsap_list_kernel<<<grid, block, smem, s>>>(a); break;
    }
    return launch_status();
}

}  // namespace

extern "C" int rfdetr_match_cost(void *stream, const void *pred_logits, int logits_dtype, const void *pred_boxes,
                                 int boxes_dtype, const int32_t *target_labels, const float *target_boxes,
                                 const uint8_t *target_mask, float *cost, int64_t batch, int64_t queries,
                                 int64_t classes, int64_t targets, float cost_class, float cost_bbox,
                                 float cost_giou, float focal_alpha) {
    return launch_match_cost(stream, pred_logits, logits_dtype, pred_boxes, boxes_dtype, target_labels, target_boxes,
                             target_mask, cost, batch, batch, queries, classes, targets, cost_class, cost_bbox,
                             cost_giou, focal_alpha);
}

extern "C" int rfdetr_lsap_batched(void *stream, const float *cost, const int32_t *sizes, int64_t problems,
                                   int64_t queries, int64_t max_targets, int64_t group_detr, int32_t *rows,
                                   int32_t *cols, uint8_t *valid, int32_t *status_out) {
    return launch_lsap(stream, cost, sizes, problems, problems, queries, max_targets, group_detr, rows, cols, valid,
                       status_out);
}

extern "C" int rfdetr_match_stacked(void *stream, const void *pred_logits, int logits_dtype, const void *pred_boxes,
                                    int boxes_dtype, const int32_t *target_labels, const float *target_boxes,
                                    const uint8_t *target_mask, const int32_t *sizes, int64_t layers, int64_t batch,
                                    int64_t queries, int64_t classes, int64_t targets, int64_t group_detr,
                                    float cost_class, float cost_bbox, float cost_giou, float focal_alpha,
                                    float *cost, int32_t *rows, int32_t *cols, uint8_t *valid, int32_t *status_out) {
    if (layers < 0 || batch < 0 || layers > 65535 || batch > 65535 || layers * batch > 65535) return RFDETR_ERR_SHAPE;
    if (layers == 0 || batch == 0) return RFDETR_OK;
    // Check the solver's limits before launching the cost.
    if (queries <= 0 || targets <= 0 || group_detr <= 0 || queries % group_detr != 0 || targets > kLsapMaxTargets ||
        queries / group_detr > kLsapMaxGroup)
        return RFDETR_ERR_SHAPE;
    if (!sizes || !rows || !cols || !valid || !status_out) return RFDETR_ERR_SHAPE;
    const int st = launch_match_cost(stream, pred_logits, logits_dtype, pred_boxes, boxes_dtype, target_labels,
                                     target_boxes, target_mask, cost, layers * batch, batch, queries, classes, targets,
                                     cost_class, cost_bbox, cost_giou, focal_alpha);
    if (st != RFDETR_OK) return st;
    return launch_lsap(stream, cost, sizes, batch, layers * batch, queries, targets, group_detr, rows, cols, valid,
                       status_out);
}
