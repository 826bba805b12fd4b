/*
 * CPU oracle for the SpMM hot path: a plain-C restatement of the reference's
 * host-side layout algorithms and of the SpMM semantics its kernels compute.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links, loads or calls this
 * file; only tests/, __graft_entry__.smoke() and the CPU-baseline leg of
 * bench.py use it, as the checker.  Parity of this restatement is pinned
 * against the reference's own compiled preprocessing (oracle/build_ref.py)
 * and against the committed golden fixtures under tests/golden/.
 *
 * Reference: IDMG-Lab/Ascend-SpMM.  Citations are path:line in that project.
 *
 * Conventions.  Indices are int64 here (the Python wrapper converts to and
 * from the caller's index dtype).  Values are opaque elements of `esz` bytes
 * that the layout functions only move, never interpret, so every value dtype
 * (f16/f32/f64) is handled bit-exactly.  Every output array is malloc'ed and
 * released by orc_free_*().  Functions return 0 on success and a non-zero
 * status with a message in orc_last_error() on invalid input.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static char g_err[256];
const char *orc_last_error(void) { return g_err; }

static int fail(const char *msg)
{
    snprintf(g_err, sizeof g_err, "%s", msg);
    return 1;
}

static void *xcalloc(int64_t n, int64_t sz)
{
    if (n <= 0) n = 1;
    return calloc((size_t)n, (size_t)sz);
}

/* ------------------------------------------------------------------------ */
/* Output containers                                                         */
/* ------------------------------------------------------------------------ */

typedef struct {
    int64_t *crow_window_ptr; int64_t n_crow;
    int64_t *unique_col_ids;  int64_t n_uniq;
    uint8_t *value;           int64_t n_value;   /* element count */
    int64_t *vrow_window_ptr; int64_t n_vrow;
    int64_t *vcol_indices;    int64_t n_vcol;
    uint8_t *vvalue;          int64_t n_vvalue;  /* element count */
} orc_layout;

typedef struct {
    orc_layout fwd;
    orc_layout tr;
    int64_t *renumbered_unique_col_ids; int64_t n_ren_uniq;
    int64_t *renumbered_vcol_indices;   int64_t n_ren_vcol;
    int64_t *permutation;               int64_t n_perm;
    int64_t *inv_permutation;           int64_t n_inv;
    int64_t packed_rows;
    int64_t packed_layout_supported;
    int64_t marginal_window;
    int64_t marginal_aic_blocks;
    int64_t marginal_total_blocks;
    int64_t shared_windows;
    double estimated_aic_cost;
    double estimated_aiv_cost;
    double estimated_max_cost;
} orc_preprocess_out;

void orc_free_layout(orc_layout *o)
{
    free(o->crow_window_ptr); free(o->unique_col_ids); free(o->value);
    free(o->vrow_window_ptr); free(o->vcol_indices); free(o->vvalue);
    memset(o, 0, sizeof *o);
}

void orc_free_preprocess(orc_preprocess_out *o)
{
    orc_free_layout(&o->fwd);
    orc_free_layout(&o->tr);
    free(o->renumbered_unique_col_ids); free(o->renumbered_vcol_indices);
    free(o->permutation); free(o->inv_permutation);
    memset(o, 0, sizeof *o);
}

static int check_csr(int64_t nrows, int64_t ncols, int64_t nnz,
                     const int64_t *crow, const int64_t *col)
{
    if (nrows < 0 || ncols < 0 || nnz < 0) return fail("negative size");
    if (crow[0] != 0 || crow[nrows] != nnz) return fail("row pointer must start at 0 and end at nnz");
    for (int64_t r = 0; r < nrows; ++r)
        if (crow[r + 1] < crow[r]) return fail("row pointer must be non-decreasing");
    for (int64_t p = 0; p < nnz; ++p)
        if (col[p] < 0 || col[p] >= ncols) return fail("column index out of range");
    return 0;
}

/* ------------------------------------------------------------------------ */
/* 16-way window merge shared by csr_to_bcsr and csr_to_ascend_cube.        */
/*                                                                          */
/* Follows the merge loop of ToBCSR (extension/custom_op.cpp:611-671) and   */
/* of the tile converter (custom_op.cpp:446-519): each row of the window    */
/* keeps a cursor; every step takes the smallest current column, the lowest */
/* row winning ties (std::min_element semantics), and emits (row, p).  An   */
/* exhausted row drops out.  The reference reads col[] one past an          */
/* exhausted row's end (custom_op.cpp:664); the cursor check here does not. */
/* ------------------------------------------------------------------------ */

typedef void (*merge_emit_fn)(void *ctx, int64_t row_in_window, int64_t col, int64_t p);

static void window_merge(const int64_t *crow, const int64_t *col, int64_t nrows,
                         int64_t w, int64_t window_size, merge_emit_fn emit, void *ctx)
{
    int64_t pos[64], end[64];
    const int64_t r0 = w * window_size;
    for (int64_t i = 0; i < window_size; ++i) {
        const int64_t r = r0 + i;
        pos[i] = end[i] = 0;
        if (r < nrows) { pos[i] = crow[r]; end[i] = crow[r + 1]; }
    }
    for (;;) {
        int64_t best = -1, best_col = 0;
        for (int64_t i = 0; i < window_size; ++i) {
            if (pos[i] >= end[i]) continue;
            if (best < 0 || col[pos[i]] < best_col) { best = i; best_col = col[pos[i]]; }
        }
        if (best < 0) break;
        emit(ctx, best, best_col, pos[best]);
        ++pos[best];
    }
}

/* ---- csr_to_bcsr: (16 x 1)-block BCSR, custom_op.cpp:594-746 ---------- */

typedef struct {
    int64_t *uniq; uint8_t *value; const uint8_t *val; int64_t esz;
    int64_t n_uniq; int64_t last;
} bcsr_ctx;

static void bcsr_emit(void *vctx, int64_t i, int64_t c, int64_t p)
{
    bcsr_ctx *x = (bcsr_ctx *)vctx;
    if (c != x->last) { x->uniq[x->n_uniq++] = c; x->last = c; }
    /* value[16 * block + row], custom_op.cpp:661 (stride is always 16) */
    memcpy(x->value + (16 * (x->n_uniq - 1) + i) * x->esz, x->val + p * x->esz, (size_t)x->esz);
}

int orc_csr_to_bcsr(int64_t nrows, int64_t ncols, int64_t nnz, const int64_t *crow,
                    const int64_t *col, const void *val, int64_t esz, int64_t window_size,
                    orc_layout *out)
{
    memset(out, 0, sizeof *out);
    if (window_size < 1 || window_size > 16) return fail("window_size must be in [1, 16]");
    if (check_csr(nrows, ncols, nnz, crow, col)) return 1;
    const int64_t nwin = (nrows + window_size - 1) / window_size;
    out->crow_window_ptr = xcalloc(nwin + 1, 8); out->n_crow = nwin + 1;
    bcsr_ctx x = { xcalloc(nnz, 8), xcalloc(16 * nnz, esz), (const uint8_t *)val, esz, 0, -1 };
    for (int64_t w = 0; w < nwin; ++w) {
        out->crow_window_ptr[w] = x.n_uniq;
        x.last = -1;
        window_merge(crow, col, nrows, w, window_size, bcsr_emit, &x);
    }
    out->crow_window_ptr[nwin] = x.n_uniq;
    out->unique_col_ids = x.uniq; out->n_uniq = x.n_uniq;
    out->value = x.value; out->n_value = 16 * x.n_uniq;
    return 0;
}

/* ---- csr_to_ascend_cube: 16 x 16 tiles, custom_op.cpp:429-592 ---------- */

typedef struct {
    int64_t *uniq; uint8_t *value; const uint8_t *val; int64_t esz;
    int64_t n_uniq; int64_t n_tile; int64_t cnt; int64_t last;
} cube_ctx;

static void cube_emit(void *vctx, int64_t i, int64_t c, int64_t p)
{
    cube_ctx *x = (cube_ctx *)vctx;
    if (c != x->last) {
        x->uniq[x->n_uniq++] = c;
        if (++x->cnt == 16) { x->cnt = 0; ++x->n_tile; }
        x->last = c;
    }
    /* value[256 * tile + 16 * row + k], custom_op.cpp:501 */
    memcpy(x->value + (256 * x->n_tile + 16 * i + x->cnt) * x->esz, x->val + p * x->esz,
           (size_t)x->esz);
}

int orc_csr_to_ascend_cube(int64_t nrows, int64_t ncols, int64_t nnz, const int64_t *crow,
                           const int64_t *col, const void *val, int64_t esz,
                           int64_t window_size, orc_layout *out)
{
    memset(out, 0, sizeof *out);
    if (window_size < 1 || window_size > 16) return fail("window_size must be in [1, 16]");
    if (check_csr(nrows, ncols, nnz, crow, col)) return 1;
    const int64_t nwin = (nrows + window_size - 1) / window_size;
    const int64_t max_tiles = nnz + nwin;
    out->crow_window_ptr = xcalloc(nwin + 1, 8); out->n_crow = nwin + 1;
    cube_ctx x = { xcalloc(16 * max_tiles, 8), xcalloc(256 * max_tiles, esz),
                   (const uint8_t *)val, esz, 0, 0, -1, -1 };
    for (int64_t w = 0; w < nwin; ++w) {
        out->crow_window_ptr[w] = x.n_tile;
        x.cnt = -1; x.last = -1;
        window_merge(crow, col, nrows, w, window_size, cube_emit, &x);
        if (x.cnt != -1) {                 /* pad the last tile, custom_op.cpp:539-543 */
            for (; x.cnt < 15; ++x.cnt) x.uniq[x.n_uniq++] = 0;
            ++x.n_tile;
        }
    }
    out->crow_window_ptr[nwin] = x.n_tile;
    out->unique_col_ids = x.uniq; out->n_uniq = 16 * x.n_tile;
    out->value = x.value; out->n_value = 256 * x.n_tile;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* block_level_split, custom_op.cpp:1146-1348 (hybrid_split_impl).           */
/* Columns inside a row need not be sorted (the graph-layout transpose      */
/* feeds unsorted rows through the same routine, custom_op.cpp:1350-1384).  */
/* ------------------------------------------------------------------------ */

static int cmp_i64(const void *a, const void *b)
{
    const int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

int orc_block_level_split(int64_t nrows, int64_t ncols, int64_t nnz, const int64_t *crow,
                          const int64_t *col, const void *valv, int64_t esz, double a,
                          int64_t window_size, orc_layout *out)
{
    memset(out, 0, sizeof *out);
    if (window_size < 1) return fail("window_size must be positive");
    if (check_csr(nrows, ncols, nnz, crow, col)) return 1;
    const uint8_t *val = (const uint8_t *)valv;
    const int64_t nwin = (nrows + window_size - 1) / window_size;
    const int64_t m_pad = nwin * window_size;

    /* Phase 1 (custom_op.cpp:1167-1192): blocks in window-major first-seen
     * order with their nonzero counts. */
    int64_t *blk_col = xcalloc(nnz, 8), *blk_cnt = xcalloc(nnz, 8);
    int64_t *win_start = xcalloc(nwin + 1, 8);
    int64_t *epoch = xcalloc(ncols, 8), *slot = xcalloc(ncols, 8);
    for (int64_t c = 0; c < ncols; ++c) epoch[c] = -1;
    int64_t nblk = 0;
    for (int64_t w = 0; w < nwin; ++w) {
        const int64_t r0 = w * window_size, r1 = r0 + window_size < nrows ? r0 + window_size : nrows;
        win_start[w] = nblk;
        for (int64_t p = crow[r0]; p < crow[r1]; ++p) {
            const int64_t c = col[p];
            if (epoch[c] != w) { epoch[c] = w; slot[c] = nblk; blk_col[nblk] = c; blk_cnt[nblk] = 0; ++nblk; }
            ++blk_cnt[slot[c]];
        }
    }
    win_start[nwin] = nblk;

    /* Phase 2 (custom_op.cpp:1197-1223): stable ascending order by count,
     * prefix sums of moved nonzeros, first k minimizing |ratio - a|.
     * Counts are small integers, so a stable counting sort gives the same
     * order as std::stable_sort. */
    int64_t maxcnt = 0;
    for (int64_t b = 0; b < nblk; ++b) if (blk_cnt[b] > maxcnt) maxcnt = blk_cnt[b];
    int64_t *bucket = xcalloc(maxcnt + 2, 8), *order = xcalloc(nblk, 8);
    for (int64_t b = 0; b < nblk; ++b) ++bucket[blk_cnt[b] + 1];
    for (int64_t k = 1; k <= maxcnt + 1; ++k) bucket[k] += bucket[k - 1];
    for (int64_t b = 0; b < nblk; ++b) order[bucket[blk_cnt[b]]++] = b;
    int64_t best_k = 0, moved_nz = 0, best_nz = 0;
    double best_diff = INFINITY;
    for (int64_t k = 0; k <= nblk; ++k) {
        if (k > 0) moved_nz += blk_cnt[order[k - 1]];
        const int64_t rem = nblk - k;
        const double ratio = moved_nz == 0 ? (rem > 0 ? INFINITY : 0.0)
                                           : (double)rem / (double)moved_nz;
        const double diff = fabs(ratio - a);
        if (diff < best_diff) { best_diff = diff; best_k = k; best_nz = moved_nz; }
    }
    char *moved = xcalloc(nblk, 1);
    for (int64_t i = 0; i < best_k; ++i) moved[order[i]] = 1;

    /* Phase 3a (custom_op.cpp:1229-1273): kept blocks, ascending columns per
     * window, zero-padded values; the last write of a (block, row) wins. */
    out->crow_window_ptr = xcalloc(nwin + 1, 8); out->n_crow = nwin + 1;
    for (int64_t w = 0; w < nwin; ++w) {
        int64_t kept = 0;
        for (int64_t b = win_start[w]; b < win_start[w + 1]; ++b) kept += !moved[b];
        out->crow_window_ptr[w + 1] = out->crow_window_ptr[w] + kept;
    }
    const int64_t n_kept = out->crow_window_ptr[nwin];
    out->unique_col_ids = xcalloc(n_kept, 8); out->n_uniq = n_kept;
    out->value = xcalloc(n_kept * window_size, esz); out->n_value = n_kept * window_size;
    for (int64_t c = 0; c < ncols; ++c) epoch[c] = -1;
    for (int64_t w = 0; w < nwin; ++w) {
        int64_t pos = out->crow_window_ptr[w];
        const int64_t base = pos;
        for (int64_t b = win_start[w]; b < win_start[w + 1]; ++b)
            if (!moved[b]) out->unique_col_ids[pos++] = blk_col[b];
        qsort(out->unique_col_ids + base, (size_t)(pos - base), 8, cmp_i64);
        for (int64_t s = base; s < pos; ++s) { epoch[out->unique_col_ids[s]] = w; slot[out->unique_col_ids[s]] = s; }
        const int64_t r0 = w * window_size, r1 = r0 + window_size < nrows ? r0 + window_size : nrows;
        for (int64_t r = r0; r < r1; ++r)
            for (int64_t p = crow[r]; p < crow[r + 1]; ++p)
                if (epoch[col[p]] == w)
                    memcpy(out->value + (slot[col[p]] * window_size + (r - r0)) * esz, val + p * esz, (size_t)esz);
    }

    /* Phase 3b (custom_op.cpp:1279-1308): CSR of the moved nonzeros over
     * m_pad rows in original order; padding rows repeat the pointer. */
    out->vrow_window_ptr = xcalloc(m_pad + 1, 8); out->n_vrow = m_pad + 1;
    out->vcol_indices = xcalloc(best_nz, 8); out->n_vcol = best_nz;
    out->vvalue = xcalloc(best_nz, esz); out->n_vvalue = best_nz;
    for (int64_t c = 0; c < ncols; ++c) epoch[c] = -1;
    int64_t vn = 0;
    for (int64_t w = 0; w < nwin; ++w) {
        for (int64_t b = win_start[w]; b < win_start[w + 1]; ++b)
            if (moved[b]) epoch[blk_col[b]] = w;
        const int64_t r0 = w * window_size;
        for (int64_t r = r0; r < r0 + window_size; ++r) {
            out->vrow_window_ptr[r] = vn;
            if (r >= nrows) continue;
            for (int64_t p = crow[r]; p < crow[r + 1]; ++p)
                if (epoch[col[p]] == w) {
                    out->vcol_indices[vn] = col[p];
                    memcpy(out->vvalue + vn * esz, val + p * esz, (size_t)esz);
                    ++vn;
                }
        }
    }
    out->vrow_window_ptr[m_pad] = vn;

    free(blk_col); free(blk_cnt); free(win_start); free(epoch); free(slot);
    free(bucket); free(order); free(moved);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* preprocess (task mapping), custom_op.cpp:765-1137.                        */
/* ------------------------------------------------------------------------ */

typedef struct { int64_t w, nnz, blocks; double density; } win_stat;

static int cmp_win(const void *a, const void *b)
{
    /* density descending, window id ascending: custom_op.cpp:808-811 */
    const win_stat *x = (const win_stat *)a, *y = (const win_stat *)b;
    if (x->density != y->density) return x->density > y->density ? -1 : 1;
    return (x->w > y->w) - (x->w < y->w);
}

int orc_preprocess(int64_t nrows, int64_t ncols, int64_t nnz, const int64_t *crow,
                   const int64_t *col, const void *valv, int64_t esz, int64_t window_size,
                   int graph_layout, orc_preprocess_out *out)
{
    memset(out, 0, sizeof *out);
    if (window_size != 16) return fail("Ascend-SpMM requires a 16-row window");
    if (check_csr(nrows, ncols, nnz, crow, col)) return 1;
    const uint8_t *val = (const uint8_t *)valv;
    const double bw_aic = 295.0, bw_aiv = 505.0;   /* custom_op.cpp:778-779 */
    const int64_t W = window_size;
    const int64_t nwin = (nrows + W - 1) / W;

    /* window statistics, custom_op.cpp:784-806 */
    win_stat *ws = xcalloc(nwin, sizeof(win_stat));
    int64_t *epoch = xcalloc(ncols, 8);
    for (int64_t c = 0; c < ncols; ++c) epoch[c] = -1;
    for (int64_t w = 0; w < nwin; ++w) {
        const int64_t r0 = w * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        int64_t blocks = 0;
        for (int64_t p = crow[r0]; p < crow[r1]; ++p)
            if (epoch[col[p]] != w) { epoch[col[p]] = w; ++blocks; }
        const int64_t wn = crow[r1] - crow[r0];
        ws[w].w = w; ws[w].nnz = wn; ws[w].blocks = blocks;
        ws[w].density = blocks ? (double)wn / (double)blocks : 0.0;
    }
    /* qsort is not stable, but (density, id) is a total order, so the
     * result equals the reference's std::stable_sort. */
    qsort(ws, (size_t)nwin, sizeof(win_stat), cmp_win);

    /* marginal-window scan, custom_op.cpp:813-826 */
    int64_t boundary_pos = -1, prefix_blocks = 0, remaining = nnz;
    for (int64_t pos = 0; pos < nwin; ++pos) {
        const double aic_after = (double)(prefix_blocks + ws[pos].blocks) / bw_aic;
        const double aiv_after = (double)(remaining - ws[pos].nnz) / bw_aiv;
        if (aic_after >= aiv_after) { boundary_pos = pos; break; }
        prefix_blocks += ws[pos].blocks;
        remaining -= ws[pos].nnz;
    }

    /* marginal-window block split, custom_op.cpp:836-885 */
    int64_t bwin = -1, bblocks = 0, baic = 0;
    double e_aic = 0.0, e_aiv = 0.0, e_max = 0.0;
    char *to_aic = xcalloc(ncols, 1);
    if (boundary_pos >= 0) {
        const win_stat *bs = &ws[boundary_pos];
        bwin = bs->w; bblocks = bs->blocks;
        int64_t *occ = xcalloc(ncols, 8), *cols = xcalloc(bblocks, 8);
        int64_t nc = 0;
        const int64_t r0 = bwin * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        for (int64_t p = crow[r0]; p < crow[r1]; ++p)
            if (occ[col[p]]++ == 0) cols[nc++] = col[p];
        /* stable bucket sort by occupancy, descending
         * (extension/boundary_bucket_sort.h:13-56); occupancy must be in
         * [1, W], i.e. no duplicate coordinates. */
        int64_t cnt_of[17] = {0};
        for (int64_t i = 0; i < nc; ++i) {
            const int64_t o = occ[cols[i]];
            if (o < 1 || o > W) {
                free(occ); free(cols); free(ws); free(epoch); free(to_aic);
                return fail("block occupancy must be in [1, window_size]; coalesce duplicate CSR entries");
            }
            ++cnt_of[o];
        }
        int64_t start_of[17], off = 0;
        for (int64_t o = W; o >= 1; --o) { start_of[o] = off; off += cnt_of[o]; }
        int64_t *sorted = xcalloc(nc, 8);
        for (int64_t i = 0; i < nc; ++i) sorted[start_of[occ[cols[i]]]++] = cols[i];
        const int64_t suffix_nnz = remaining - bs->nnz;
        int64_t assigned = 0, best_q = 0;
        double best = INFINITY;
        for (int64_t q = 0; q <= bblocks; ++q) {
            const double ac = (double)(prefix_blocks + q) / bw_aic;
            const double vc = (double)(suffix_nnz + bs->nnz - assigned) / bw_aiv;
            const double mc = ac > vc ? ac : vc;
            if (mc < best) { best = mc; best_q = q; e_aic = ac; e_aiv = vc; e_max = mc; }
            if (q < bblocks) assigned += occ[sorted[q]];
        }
        baic = best_q;
        for (int64_t q = 0; q < best_q; ++q) to_aic[sorted[q]] = 1;
        free(occ); free(cols); free(sorted);
    }

    /* window lists, custom_op.cpp:887-903 */
    int64_t *aic = xcalloc(nwin, 8), *aiv = xcalloc(nwin, 8);
    int64_t naic = 0, naiv = 0;
    if (boundary_pos < 0) {
        for (int64_t i = 0; i < nwin; ++i) aiv[naiv++] = ws[i].w;
    } else {
        for (int64_t i = 0; i < boundary_pos; ++i) aic[naic++] = ws[i].w;
        if (baic > 0) aic[naic++] = bwin; else aiv[naiv++] = bwin;
        for (int64_t i = boundary_pos + 1; i < nwin; ++i) aiv[naiv++] = ws[i].w;
    }

    /* row permutation, custom_op.cpp:905-940 */
    const int shared = baic > 0 && baic < bblocks;
    const int64_t aic_pad_rows = naic * W;
    int64_t aic_real_rows = 0;
    for (int64_t s = 0; s < naic; ++s) {
        const int64_t r0 = aic[s] * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        aic_real_rows += r1 - r0;
    }
    const int64_t real_extent = aic_pad_rows + (nrows - aic_real_rows);
    const int64_t packed_ok = (graph_layout && nrows == ncols) ? 1 : 0;
    const int64_t out_rows = packed_ok ? nwin * W : real_extent;
    int64_t *perm = xcalloc(out_rows, 8), *inv = xcalloc(nrows, 8);
    for (int64_t i = 0; i < out_rows; ++i) perm[i] = -1;
    for (int64_t i = 0; i < nrows; ++i) inv[i] = -1;
    for (int64_t s = 0; s < naic; ++s) {
        const int64_t r0 = aic[s] * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        for (int64_t r = r0; r < r1; ++r) { perm[s * W + (r - r0)] = r; inv[r] = s * W + (r - r0); }
    }
    int64_t vrow = aic_pad_rows;
    for (int64_t i = 0; i < naiv; ++i) {
        const int64_t r0 = aiv[i] * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        for (int64_t r = r0; r < r1; ++r) { perm[vrow] = r; inv[r] = vrow; ++vrow; }
    }

    /* AIC pack, custom_op.cpp:942-979: per slot, ascending distinct columns
     * (minus the marginal window's AIV columns when it is shared). */
    orc_layout *f = &out->fwd;
    f->crow_window_ptr = xcalloc(naic + 1, 8); f->n_crow = naic + 1;
    int64_t total_blocks = 0;
    for (int64_t c = 0; c < ncols; ++c) epoch[c] = -1;
    for (int64_t s = 0; s < naic; ++s) {
        const int64_t w = aic[s], r0 = w * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        for (int64_t p = crow[r0]; p < crow[r1]; ++p) {
            const int64_t c = col[p];
            if (shared && w == bwin && !to_aic[c]) continue;
            if (epoch[c] != s) { epoch[c] = s; ++total_blocks; }
        }
    }
    f->unique_col_ids = xcalloc(total_blocks, 8); f->n_uniq = total_blocks;
    f->value = xcalloc(total_blocks * W, esz); f->n_value = total_blocks * W;
    int64_t *slot = xcalloc(ncols, 8);
    for (int64_t c = 0; c < ncols; ++c) epoch[c] = -1;
    int64_t nb = 0;
    for (int64_t s = 0; s < naic; ++s) {
        const int64_t w = aic[s], r0 = w * W, r1 = r0 + W < nrows ? r0 + W : nrows;
        const int64_t base = nb;
        for (int64_t p = crow[r0]; p < crow[r1]; ++p) {
            const int64_t c = col[p];
            if (shared && w == bwin && !to_aic[c]) continue;
            if (epoch[c] != s) { epoch[c] = s; f->unique_col_ids[nb++] = c; }
        }
        qsort(f->unique_col_ids + base, (size_t)(nb - base), 8, cmp_i64);
        for (int64_t b = base; b < nb; ++b) slot[f->unique_col_ids[b]] = b;
        for (int64_t r = r0; r < r1; ++r)
            for (int64_t p = crow[r]; p < crow[r + 1]; ++p) {
                const int64_t c = col[p];
                if (shared && w == bwin && !to_aic[c]) continue;
                memcpy(f->value + (slot[c] * W + (r - r0)) * esz, val + p * esz, (size_t)esz);
            }
        f->crow_window_ptr[s + 1] = nb;
    }

    /* AIV pack over packed rows, custom_op.cpp:981-1001 */
    f->vrow_window_ptr = xcalloc(out_rows + 1, 8); f->n_vrow = out_rows + 1;
    f->vcol_indices = xcalloc(nnz, 8);
    f->vvalue = xcalloc(nnz, esz);
    int64_t vn = 0;
    for (int64_t o = 0; o < out_rows; ++o) {
        f->vrow_window_ptr[o] = vn;
        const int64_t r = perm[o];
        if (r < 0) continue;
        const int vector_owned = o >= aic_pad_rows;
        const int residual = shared && (r / W) == bwin;
        if (!vector_owned && !residual) continue;
        for (int64_t p = crow[r]; p < crow[r + 1]; ++p) {
            if (residual && to_aic[col[p]]) continue;
            f->vcol_indices[vn] = col[p];
            memcpy(f->vvalue + vn * esz, val + p * esz, (size_t)esz);
            ++vn;
        }
    }
    f->vrow_window_ptr[out_rows] = vn;
    f->n_vcol = vn; f->n_vvalue = vn;

    /* graph layout: P*A*P^T relabel + fixed-layout transpose,
     * custom_op.cpp:1006-1035, extension/packed_column_reindex.h:14-101 */
    if (packed_ok) {
        out->renumbered_unique_col_ids = xcalloc(f->n_uniq, 8); out->n_ren_uniq = f->n_uniq;
        for (int64_t i = 0; i < f->n_uniq; ++i) out->renumbered_unique_col_ids[i] = inv[f->unique_col_ids[i]];
        out->renumbered_vcol_indices = xcalloc(vn, 8); out->n_ren_vcol = vn;
        for (int64_t i = 0; i < vn; ++i) out->renumbered_vcol_indices[i] = inv[f->vcol_indices[i]];
        /* counting-sort transpose into packed ids, stable in original row order */
        int64_t *tp = xcalloc(out_rows + 1, 8), *tc = xcalloc(nnz, 8);
        uint8_t *tv = xcalloc(nnz, esz);
        for (int64_t p = 0; p < nnz; ++p) ++tp[inv[col[p]] + 1];
        for (int64_t i = 0; i < out_rows; ++i) tp[i + 1] += tp[i];
        int64_t *next = xcalloc(out_rows + 1, 8);
        memcpy(next, tp, (size_t)(out_rows + 1) * 8);
        for (int64_t r = 0; r < nrows; ++r)
            for (int64_t p = crow[r]; p < crow[r + 1]; ++p) {
                const int64_t d = next[inv[col[p]]]++;
                tc[d] = inv[r];
                memcpy(tv + d * esz, val + p * esz, (size_t)esz);
            }
        int rc = orc_block_level_split(out_rows, out_rows, nnz, tp, tc, tv, esz, 295.0 / 505.0, W, &out->tr);
        free(tp); free(tc); free(tv); free(next);
        if (rc) { free(ws); free(epoch); free(to_aic); free(aic); free(aiv); free(slot); free(perm); free(inv); return rc; }
    }

    out->permutation = perm; out->n_perm = out_rows;
    out->inv_permutation = inv; out->n_inv = nrows;
    out->packed_rows = out_rows;
    out->packed_layout_supported = packed_ok;
    out->marginal_window = bwin;
    out->marginal_aic_blocks = baic;
    out->marginal_total_blocks = bblocks;
    out->shared_windows = shared ? 1 : 0;
    out->estimated_aic_cost = e_aic;
    out->estimated_aiv_cost = e_aiv;
    out->estimated_max_cost = e_max;
    free(ws); free(epoch); free(to_aic); free(aic); free(aiv); free(slot);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* SpMM semantics in float64.                                                */
/* ------------------------------------------------------------------------ */

/* y[r, :] = sum_p val[p] * B[col[p], :]  (op_kernel/spmm_csr.cpp:383-423).
 * y must hold nrows * n zeros on entry. */
void orc_spmm_csr_f64(int64_t nrows, int64_t n, const int64_t *crow, const int64_t *col,
                      const double *val, const double *B, double *y)
{
    for (int64_t r = 0; r < nrows; ++r) {
        double *yr = y + r * n;
        for (int64_t p = crow[r]; p < crow[r + 1]; ++p) {
            const double v = val[p];
            const double *b = B + col[p] * n;
            for (int64_t j = 0; j < n; ++j) yr[j] += v * b[j];
        }
    }
}

/* Window part of the mixed operator (op_kernel/spmm_ascend_cube.cpp:52-165,
 * 265-288): window slot s adds sum_b Cvalue[16b + i] * B[Ccol[b], :] to
 * output row 16s + i.  y must be zero or hold a partial result on entry. */
void orc_spmm_window_f64(int64_t nwin, int64_t n, const int64_t *cptr, const int64_t *ccol,
                         const double *cval, const double *B, double *y)
{
    for (int64_t s = 0; s < nwin; ++s)
        for (int64_t b = cptr[s]; b < cptr[s + 1]; ++b) {
            const double *brow = B + ccol[b] * n;
            for (int64_t i = 0; i < 16; ++i) {
                const double v = cval[16 * b + i];
                if (v == 0.0) continue;
                double *yr = y + (16 * s + i) * n;
                for (int64_t j = 0; j < n; ++j) yr[j] += v * brow[j];
            }
        }
}

/* ------------------------------------------------------------------------ */
/* spmm_cube: window entries encoded as (column << 4) | row.                 */
/* ------------------------------------------------------------------------ */

/* The reference kernel (kernels/op_kernel/spmm_cube.cpp:51-147) walks the
 * entries of window w = [rowptr[w], rowptr[w+1]) in order.  An entry whose
 * column (col >> 4) differs from the previous entry's opens a new (16 x 1)
 * block (spmm_cube.cpp:88-107; the first entry of a window always does,
 * :77); the entry's value is stored at row (col & 15) of that block,
 * overwriting an earlier entry of the same row in the same block (:125-126).
 * Every block adds block[r] * B[column, :] to output row 16 w + r
 * (:210, :235-236).  y must hold 16 * nwin * n zeros on entry. */
void orc_spmm_cube_f64(int64_t nwin, int64_t n, const int64_t *rowptr, const int64_t *col,
                       const double *val, const double *B, double *y)
{
    double a[16];
    int set[16];
    for (int64_t w = 0; w < nwin; ++w) {
        int64_t cur = 0;
        int open = 0;
        for (int64_t p = rowptr[w]; p <= rowptr[w + 1]; ++p) {
            const int end = p == rowptr[w + 1];
            const int64_t c = end ? 0 : (col[p] >> 4);
            if (open && (end || c != cur)) {
                const double *brow = B + cur * n;
                for (int r = 0; r < 16; ++r) {
                    if (!set[r]) continue;
                    double *yr = y + (16 * w + r) * n;
                    for (int64_t j = 0; j < n; ++j) yr[j] += a[r] * brow[j];
                }
                open = 0;
            }
            if (end) break;
            if (!open) {
                memset(set, 0, sizeof set);
                cur = c;
                open = 1;
            }
            a[col[p] & 15] = val[p];
            set[col[p] & 15] = 1;
        }
    }
}

/* Producer of that encoding (the reference ships the consumer only): per
 * 16-row window, the window's entries ordered by (column, row), entries of
 * equal (column, row) in CSR position order - the order in which ToBCSR's
 * 16-way merge visits a window with sorted rows (custom_op.cpp:611-671), so
 * every run of equal columns is one (16 x 1) block of csr_to_bcsr and the
 * last duplicate wins in both.  Output: crow_window_ptr [nwin + 1] (entry
 * offsets, = crow[min(16 w, nrows)]), unique_col_ids [nnz] holding
 * (column << 4) | row, value [nnz]. */
typedef struct { int64_t key, p; } cube_ent;

static int cmp_cube_ent(const void *x, const void *y)
{
    const cube_ent *a = (const cube_ent *)x, *b = (const cube_ent *)y;
    if (a->key != b->key) return a->key < b->key ? -1 : 1;
    return a->p < b->p ? -1 : (a->p > b->p);
}

int orc_csr_to_spmm_cube(int64_t nrows, int64_t ncols, int64_t nnz, const int64_t *crow,
                         const int64_t *col, const void *val, int64_t esz, int64_t window_size,
                         orc_layout *out)
{
    memset(out, 0, sizeof *out);
    if (window_size != 16) return fail("window_size must be 16");
    if (check_csr(nrows, ncols, nnz, crow, col)) return 1;
    const int64_t nwin = (nrows + 15) / 16;
    out->crow_window_ptr = (int64_t *)xcalloc(nwin + 1, sizeof(int64_t));
    out->unique_col_ids = (int64_t *)xcalloc(nnz, sizeof(int64_t));
    out->value = (uint8_t *)xcalloc(nnz, esz);
    cube_ent *e = (cube_ent *)xcalloc(nnz, sizeof(cube_ent));
    if (!out->crow_window_ptr || !out->unique_col_ids || !out->value || !e) {
        free(e);
        orc_free_layout(out);
        return fail("out of memory");
    }
    out->n_crow = nwin + 1;
    out->n_uniq = out->n_value = nnz;
    const uint8_t *v = (const uint8_t *)val;
    for (int64_t w = 0; w <= nwin; ++w) out->crow_window_ptr[w] = crow[w * 16 < nrows ? w * 16 : nrows];
    for (int64_t w = 0; w < nwin; ++w) {
        const int64_t p0 = out->crow_window_ptr[w], p1 = out->crow_window_ptr[w + 1];
        for (int64_t r = 16 * w; r < 16 * w + 16 && r < nrows; ++r)
            for (int64_t p = crow[r]; p < crow[r + 1]; ++p) {
                e[p].key = (col[p] << 4) | (r & 15);
                e[p].p = p;
            }
        qsort(e + p0, (size_t)(p1 - p0), sizeof(cube_ent), cmp_cube_ent);
        for (int64_t q = p0; q < p1; ++q) {
            out->unique_col_ids[q] = e[q].key;
            memcpy(out->value + q * esz, v + e[q].p * esz, (size_t)esz);
        }
    }
    free(e);
    return 0;
}
