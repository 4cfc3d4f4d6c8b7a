/*
 * CPU restatement of SciPy's linear_sum_assignment -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * The reference solves every (image, group) block with scipy.optimize.linear_sum_assignment
 * (src/rfdetr_jax/models/matcher.py:27,173).  SciPy (>= 1.4; 1.18.1 installed here) implements
 * the shortest-augmenting-path method of D. F. Crouse, "On implementing 2D rectangular
 * assignment algorithms", IEEE Trans. Aerospace and Electronic Systems 52(4), 2016, in float64.
 * This file restates that published method, with the choices that decide ties:
 *
 *   - a tall matrix (more rows than columns) is solved transposed, and the answer is
 *     reported sorted by the original row index;
 *   - rows are inserted in index order; each insertion runs a Dijkstra-like search over the
 *     columns that are not yet scanned, visited through a work list that starts in descending
 *     column order and drops a scanned column by moving the list's last entry into its slot;
 *   - reduced costs are evaluated as ((minVal + c[i][j]) - u[i]) - v[j];
 *   - the next column is the one with the smallest tentative distance; among equal distances
 *     an unassigned column is preferred, the later one in the work list if several are
 *     unassigned, otherwise the earliest one in the work list;
 *   - duals: u[cur] += minVal; u[i] += minVal - d[col4row[i]] for the other scanned rows;
 *     v[j] -= minVal - d[j] for scanned columns; then the path is flipped back to cur.
 *
 * It exists to be checked bit-exactly against SciPy (tests/test_oracle_lsap_topk.py), which pins
 * the tie rules that the CUDA solver reproduces.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Returns 0 on success, -1 for invalid entries (NaN or -inf), -2 if infeasible. */
int oracle_lsap(int64_t nr, int64_t nc, const double *input, int64_t *rows_out, int64_t *cols_out)
{
    if (nr <= 0 || nc <= 0) return 0;
    int transpose = nc < nr;
    double *cost = (double *)malloc(sizeof(double) * (size_t)(nr * nc));
    if (!cost) return -3;
    if (transpose) {
        for (int64_t i = 0; i < nr; ++i)
            for (int64_t j = 0; j < nc; ++j) cost[j * nr + i] = input[i * nc + j];
        int64_t t = nr; nr = nc; nc = t;
    } else {
        memcpy(cost, input, sizeof(double) * (size_t)(nr * nc));
    }
    for (int64_t k = 0; k < nr * nc; ++k) {
        if (cost[k] != cost[k] || cost[k] == -INFINITY) { free(cost); return -1; }
    }

    double *u = (double *)calloc((size_t)nr, sizeof(double));
    double *v = (double *)calloc((size_t)nc, sizeof(double));
    double *dist = (double *)malloc(sizeof(double) * (size_t)nc);
    int64_t *path = (int64_t *)malloc(sizeof(int64_t) * (size_t)nc);
    int64_t *col4row = (int64_t *)malloc(sizeof(int64_t) * (size_t)nr);
    int64_t *row4col = (int64_t *)malloc(sizeof(int64_t) * (size_t)nc);
    char *row_seen = (char *)malloc((size_t)nr);
    char *col_seen = (char *)malloc((size_t)nc);
    int64_t *todo = (int64_t *)malloc(sizeof(int64_t) * (size_t)nc);
    for (int64_t j = 0; j < nc; ++j) { path[j] = -1; row4col[j] = -1; }
    for (int64_t i = 0; i < nr; ++i) col4row[i] = -1;
    int status = 0;

    for (int64_t cur = 0; cur < nr && status == 0; ++cur) {
        double min_val = 0.0;
        int64_t left = nc;
        for (int64_t k = 0; k < nc; ++k) todo[k] = nc - 1 - k;
        memset(row_seen, 0, (size_t)nr);
        memset(col_seen, 0, (size_t)nc);
        for (int64_t j = 0; j < nc; ++j) dist[j] = INFINITY;

        int64_t i = cur, sink = -1;
        while (sink == -1) {
            int64_t pick = -1;
            double lowest = INFINITY;
            row_seen[i] = 1;
            for (int64_t k = 0; k < left; ++k) {
                int64_t j = todo[k];
                double r = min_val + cost[i * nc + j] - u[i] - v[j];
                if (r < dist[j]) { path[j] = i; dist[j] = r; }
                if (dist[j] < lowest || (dist[j] == lowest && row4col[j] == -1)) {
                    lowest = dist[j];
                    pick = k;
                }
            }
            min_val = lowest;
            if (min_val == INFINITY) { status = -2; break; }
            int64_t j = todo[pick];
            if (row4col[j] == -1) sink = j; else i = row4col[j];
            col_seen[j] = 1;
            todo[pick] = todo[--left];
        }
        if (status) break;

        u[cur] += min_val;
        for (int64_t r = 0; r < nr; ++r)
            if (row_seen[r] && r != cur) u[r] += min_val - dist[col4row[r]];
        for (int64_t c = 0; c < nc; ++c)
            if (col_seen[c]) v[c] -= min_val - dist[c];

        int64_t j = sink;
        for (;;) {
            int64_t r = path[j];
            row4col[j] = r;
            int64_t t = col4row[r]; col4row[r] = j; j = t;
            if (r == cur) break;
        }
    }

    if (status == 0) {
        if (transpose) {
            /* Report in original-row order: the original rows are the columns here. */
            int64_t k = 0;
            for (int64_t c = 0; c < nc; ++c) {
                if (row4col[c] >= 0) { rows_out[k] = c; cols_out[k] = row4col[c]; ++k; }
            }
        } else {
            for (int64_t r = 0; r < nr; ++r) { rows_out[r] = r; cols_out[r] = col4row[r]; }
        }
    }
    free(cost); free(u); free(v); free(dist); free(path); free(col4row); free(row4col);
    free(row_seen); free(col_seen); free(todo);
    return status;
}
