/*
 * oracle.c -- CPU restatement of the reference's binary-logloss hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA engine:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load liboracle.so.  The product path never calls it.
 *
 * Everything here restates src/bsscl_gbm/estimator_v1_0_1.py of the
 * reference (cited as E:<line>) in plain C, compiled with
 * -ffp-contract=off so every double operation rounds exactly like the
 * reference's Numba code (no fastmath on the builders, E:232, E:516).
 *
 * Two accumulation modes for the tree builders:
 *   OR_MODE_REF   -- f64 sums in the reference's own order: per-feature
 *                    sequential sums over the node's rows in index order,
 *                    the larger child's histogram by f64 subtraction
 *                    (E:582-596, E:723-745).  Bit-exact with the reference;
 *                    pinned by tests/golden.
 *   OR_MODE_EXACT -- the CUDA engine's semantics: every g/h is rounded once
 *                    to the fixed-point grid 2^-S (S = `scale_bits`), all
 *                    sums are exact integer sums (order independent), and
 *                    each sum is converted to f64 once.  The GPU must match
 *                    this mode bit-for-bit.
 *   Mode EXACT uses 128-bit integer accumulators; the GPU keeps the same
 *   value as a pair of 64-bit words.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef __int128 i128;

enum { OR_MODE_REF = 0, OR_MODE_EXACT = 1 };

/* ------------------------------------------------------------------ */
/* Binning: E:155-226 (per-value search) and E:2144-2189 (NaN driver). */
/* ------------------------------------------------------------------ */

/* Largest k in [0, nb-1] with edge[k] <= v, after the two early outs
 * (v < edge[0] -> 0, v >= edge[nb] -> nb-1).  E:204-226. */
static int bin_standard(const double *e, int nb, double v) {
    if (v < e[0]) return 0;
    if (v >= e[nb]) return nb - 1;
    int lo = 0, hi = nb - 1;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (e[mid + 1] <= v) lo = mid + 1; else hi = mid;
    }
    return lo;
}

/* Interpolation guess, +-4 window, then full search.  E:155-202.
 * All three paths return the same id as bin_standard for non-NaN v; the
 * window/guess only changes the work done, except for NaN inputs (which
 * the driver never passes when a NaN bin exists). */
static int bin_hybrid(const double *e, int nb, double v) {
    int last = nb - 1;
    double b0 = e[0], b1 = e[nb];
    double scale = (b1 > b0) ? (double)last / (b1 - b0) : 1.0;
    if (v < b0) return 0;
    if (v >= b1) return last;
    double t = (v - b0) * scale;
    long long gi;
    if (t != t) gi = INT64_MIN;            /* int(NaN): x86 cvttsd2si result */
    else if (t >= 9.2e18) gi = INT64_MAX;
    else if (t <= -9.2e18) gi = INT64_MIN;
    else gi = (long long)t;
    int g;
    if (gi < 0) g = 0; else if (gi > last) g = last; else g = (int)gi;
    if (e[g] <= v && (g == last || v < e[g + 1])) return g;
    int lo = g - 4 < 0 ? 0 : g - 4;
    int hi = g + 4 > last ? last : g + 4;
    if (!(v >= e[lo] && (hi == last || v < e[hi + 1]))) { lo = 0; hi = last; }
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (e[mid + 1] <= v) lo = mid + 1; else hi = mid;
    }
    return lo;
}

/* X [n][p] row-major doubles (float32 inputs are widened first, which is
 * what Numba does when it compares a float32 with a float64 edge).
 * edges [p][max_b].  has_any_nan mirrors E:2157: NaN is replaced by 0.0,
 * binned, then NaN-aware features shift by +1 and NaN -> 0 (E:2174-2177). */
int or_bin_matrix(const double *X, int64_t n, int32_t p, const double *edges,
                  int32_t max_b, const int32_t *counts, const int32_t *nan_bin_id,
                  int32_t has_any_nan, int32_t hybrid, uint16_t *out) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        for (int j = 0; j < p; j++) {
            double v = X[i * p + j];
            int isnan_v = (v != v);
            if (has_any_nan && isnan_v) v = 0.0;
            const double *e = edges + (int64_t)j * max_b;
            int nb = counts[j];
            int b = hybrid ? bin_hybrid(e, nb, v) : bin_standard(e, nb, v);
            if (has_any_nan && nan_bin_id[j] >= 0) b = isnan_v ? 0 : b + 1;
            out[i * p + j] = (uint16_t)b;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Shared helpers for the tree builders.                               */
/* ------------------------------------------------------------------ */

typedef struct {
    int mode;
    int scale_bits;          /* S for OR_MODE_EXACT */
    double lam, mcw, gamma;
    int msl, max_depth, max_leaves;
} params_t;

typedef struct {            /* a histogram set for one node */
    double *G, *H;           /* REF:   [p][max_bins] f64            */
    i128 *QG, *QH;           /* EXACT: [p][max_bins] exact integers */
} hist_t;

static inline i128 quant(double x, int S) {
    /* round-to-nearest-even onto the 2^-S grid (exact scaling by 2^S) */
    return (i128)rint(ldexp(x, S));
}

/* int128 -> double, round to nearest even. */
static double i128_to_double(i128 v) {
    return (double)v;   /* libgcc __floattidf rounds to nearest */
}

static inline double qd(i128 v, int S) { return ldexp(i128_to_double(v), -S); }

typedef struct { int feat; int bin; double gain; int nr; } split_t;

/* The learned NaN direction (the engine's gbm_params.nan_direction; no
 * reference counterpart): when set, nanf[j] != 0 marks the features whose
 * bin 0 is the NaN bin, the split scan also evaluates at every bin t >= 1
 * the split that sends NaN right (left = bins 1..t), right after the
 * NaN-left candidate of the same bin (so NaN-left wins a tie), and a
 * tree's thresholds carry the direction in bit 32 of tt.  NULL: the
 * reference's NaN-left only. */
static const uint8_t *g_nanf = NULL;
void or_set_nan_dir(const uint8_t *nanf) { g_nanf = nanf; }

static inline int goes_left(int64_t b, int64_t thr, int nr) { return b <= thr && !(nr && b == 0); }

/* Split scan of one node's histogram.  E:602-621 / E:780-801: features in
 * ascending feature_indices order, bins 0..nb-2 as a running prefix, skip
 * HL<mcw or HR<mcw, strict '>' against an incumbent starting at -1e9. */
static split_t find_split(const params_t *P, const hist_t *hs, int max_bins,
                          const int32_t *fidx, int nf, const int32_t *counts,
                          i128 qG, i128 qH) {
    split_t best = { -1, 0, -1e9, 0 };
    for (int jj = 0; jj < nf; jj++) {
        int j = fidx[jj];
        int nb = counts[j];
        if (nb < 2) continue;
        if (P->mode == OR_MODE_REF) {
            const double *G = hs->G + (int64_t)j * max_bins, *H = hs->H + (int64_t)j * max_bins;
            double Gt = 0.0, Ht = 0.0;
            for (int b = 0; b < nb; b++) { Gt += G[b]; Ht += H[b]; }
            double GL = 0.0, HL = 0.0;
            const int nd_ = g_nanf && g_nanf[j];
            for (int b = 0; b < nb - 1; b++) {
                GL += G[b]; HL += H[b];
                for (int dir = 0; dir <= (nd_ && b >= 1); dir++) {
                    double gl_ = dir ? GL - G[0] : GL, hl_ = dir ? HL - H[0] : HL;
                    double GR = Gt - gl_, HR = Ht - hl_;
                    if (hl_ < P->mcw || HR < P->mcw) continue;
                    double gain = gl_ * gl_ / (hl_ + P->lam) + GR * GR / (HR + P->lam)
                                - Gt * Gt / (Ht + P->lam);
                    if (gain > best.gain) { best.gain = gain; best.feat = j; best.bin = b; best.nr = dir; }
                }
            }
        } else {
            const i128 *G = hs->QG + (int64_t)j * max_bins, *H = hs->QH + (int64_t)j * max_bins;
            int S = P->scale_bits;
            double Gt = qd(qG, S), Ht = qd(qH, S);
            double parent = Gt * Gt / (Ht + P->lam);
            i128 gl = 0, hl = 0;
            const int nd_ = g_nanf && g_nanf[j];
            for (int b = 0; b < nb - 1; b++) {
                gl += G[b]; hl += H[b];
                for (int dir = 0; dir <= (nd_ && b >= 1); dir++) {
                    i128 gl_ = dir ? gl - G[0] : gl, hl_ = dir ? hl - H[0] : hl;
                    double GL = qd(gl_, S), HL = qd(hl_, S);
                    double GR = qd(qG - gl_, S), HR = qd(qH - hl_, S);
                    if (HL < P->mcw || HR < P->mcw) continue;
                    double gain = GL * GL / (HL + P->lam) + GR * GR / (HR + P->lam) - parent;
                    if (gain > best.gain) { best.gain = gain; best.feat = j; best.bin = b; best.nr = dir; }
                }
            }
        }
    }
    return best;
}

/* Histogram of rows idx[a..b) into hs (features fidx only).  E:582-596. */
static void build_hist(const params_t *P, hist_t *hs, int max_bins, const uint16_t *Xb,
                       int p, const double *g, const double *h, const i128 *qg,
                       const i128 *qh, const int64_t *idx, int64_t a, int64_t b,
                       const int32_t *fidx, int nf, const int32_t *counts) {
    #pragma omp parallel for schedule(dynamic, 1)
    for (int jj = 0; jj < nf; jj++) {
        int j = fidx[jj];
        int nb = counts[j];
        if (P->mode == OR_MODE_REF) {
            double *G = hs->G + (int64_t)j * max_bins, *H = hs->H + (int64_t)j * max_bins;
            for (int k = 0; k < nb; k++) { G[k] = 0.0; H[k] = 0.0; }
            for (int64_t k = a; k < b; k++) {
                int64_t i = idx[k];
                int bv = Xb[i * p + j];
                if (bv >= nb) bv = nb - 1;
                G[bv] += g[i]; H[bv] += h[i];
            }
        } else {
            i128 *G = hs->QG + (int64_t)j * max_bins, *H = hs->QH + (int64_t)j * max_bins;
            for (int k = 0; k < nb; k++) { G[k] = 0; H[k] = 0; }
            for (int64_t k = a; k < b; k++) {
                int64_t i = idx[k];
                int bv = Xb[i * p + j];
                if (bv >= nb) bv = nb - 1;
                G[bv] += qg[i]; H[bv] += qh[i];
            }
        }
    }
}

/* dst = par - small (the sibling-subtraction trick, E:740-745). */
static void subtract_hist(const params_t *P, hist_t *dst, const hist_t *par, const hist_t *sm,
                          int max_bins, const int32_t *fidx, int nf, const int32_t *counts) {
    for (int jj = 0; jj < nf; jj++) {
        int j = fidx[jj];
        int64_t o = (int64_t)j * max_bins;
        for (int k = 0; k < counts[j]; k++) {
            if (P->mode == OR_MODE_REF) {
                dst->G[o + k] = par->G[o + k] - sm->G[o + k];
                dst->H[o + k] = par->H[o + k] - sm->H[o + k];
            } else {
                dst->QG[o + k] = par->QG[o + k] - sm->QG[o + k];
                dst->QH[o + k] = par->QH[o + k] - sm->QH[o + k];
            }
        }
    }
}

/* Node sums over idx[a..b): REF = sequential f64 (E:567-573, E:764-769);
 * EXACT = integer sums. */
static void node_sums(const params_t *P, const double *g, const double *h, const i128 *qg,
                      const i128 *qh, const int64_t *idx, int64_t a, int64_t b,
                      double *Gs, double *Hs, i128 *qG, i128 *qH) {
    if (P->mode == OR_MODE_REF) {
        double gs = 0.0, hs = 0.0;
        for (int64_t k = a; k < b; k++) { gs += g[idx[k]]; hs += h[idx[k]]; }
        *Gs = gs; *Hs = hs; *qG = 0; *qH = 0;
    } else {
        i128 gs = 0, hs = 0;
        for (int64_t k = a; k < b; k++) { gs += qg[idx[k]]; hs += qh[idx[k]]; }
        *qG = gs; *qH = hs;
        *Gs = qd(gs, P->scale_bits); *Hs = qd(hs, P->scale_bits);
    }
}

/* In-place two-pointer partition of idx[a..b) on Xb[:, f] <= thr
 * (E:663-674), NaN bin right when nr.  Returns the split position. */
static int64_t partition(int64_t *idx, int64_t a, int64_t b, const uint16_t *Xb, int p,
                         int f, int64_t thr, int nr) {
    int64_t lp = a, rp = b - 1;
    while (lp <= rp) {
        int64_t i = idx[lp];
        if (goes_left(Xb[i * p + f], thr, nr)) lp++;
        else { idx[lp] = idx[rp]; idx[rp] = i; rp--; }
    }
    return lp;
}

static int alloc_hist(hist_t *hs, int mode, int p, int max_bins) {
    size_t cells = (size_t)p * max_bins;
    hs->G = hs->H = NULL; hs->QG = hs->QH = NULL;
    if (mode == OR_MODE_REF) {
        hs->G = calloc(cells, sizeof(double)); hs->H = calloc(cells, sizeof(double));
        return hs->G && hs->H ? 0 : -1;
    }
    hs->QG = calloc(cells, sizeof(i128)); hs->QH = calloc(cells, sizeof(i128));
    return hs->QG && hs->QH ? 0 : -1;
}
static void free_hist(hist_t *hs) { free(hs->G); free(hs->H); free(hs->QG); free(hs->QH); }

static void quantize_all(const params_t *P, const double *g, const double *h, int64_t n_all,
                         i128 **qg, i128 **qh) {
    *qg = *qh = NULL;
    if (P->mode != OR_MODE_EXACT) return;
    *qg = malloc(sizeof(i128) * (size_t)n_all);
    *qh = malloc(sizeof(i128) * (size_t)n_all);
    for (int64_t i = 0; i < n_all; i++) {
        (*qg)[i] = quant(g[i], P->scale_bits);
        (*qh)[i] = quant(h[i], P->scale_bits);
    }
}

/* ------------------------------------------------------------------ */
/* Leaf-wise (best-first) builder: E:517-823.                          */
/* Outputs have 2*max_leaves+2 entries.  node_of_pos (optional, length  */
/* n_sub) receives, for each position of the final index order, the     */
/* node id whose segment holds it; idx_out receives that order.         */
/* ------------------------------------------------------------------ */
int or_build_leafwise(const uint16_t *Xb, int64_t n_all, int32_t p, const double *g,
                      const double *h, const int64_t *sample_idx, int64_t n_sub,
                      const int32_t *fidx, int32_t nf, const int32_t *counts,
                      int32_t max_bins, int32_t max_leaves, int32_t max_depth,
                      int32_t msl, double mcw, double lam, double gamma,
                      int32_t mode, int32_t scale_bits,
                      int32_t *tf, int64_t *tt, double *tv, int32_t *tl, int32_t *tr,
                      double *sg, int32_t *n_nodes) {
    params_t P = { mode, scale_bits, lam, mcw, gamma, msl, max_depth, max_leaves };
    int max_nodes = max_leaves * 2 + 2;
    for (int k = 0; k < max_nodes; k++) { tf[k] = -1; tt[k] = 0; tv[k] = 0.0; tl[k] = -1; tr[k] = -1; sg[k] = 0.0; }
    int node_count = 0;
    int64_t *idx = malloc(sizeof(int64_t) * (size_t)(n_sub > 0 ? n_sub : 1));
    memcpy(idx, sample_idx, sizeof(int64_t) * (size_t)n_sub);
    i128 *qg, *qh;
    quantize_all(&P, g, h, n_all, &qg, &qh);

    int MAX_C = max_leaves + 2;
    hist_t *hs = calloc((size_t)MAX_C, sizeof(hist_t));
    int32_t *c_node = calloc(MAX_C, 4), *c_depth = calloc(MAX_C, 4), *c_feat = calloc(MAX_C, 4);
    int32_t *c_bin = calloc(MAX_C, 4); int8_t *c_active = calloc(MAX_C, 1);
    int64_t *c_start = calloc(MAX_C, 8), *c_end = calloc(MAX_C, 8);
    double *c_gain = calloc(MAX_C, 8), *c_val = calloc(MAX_C, 8);
    i128 *c_qG = calloc(MAX_C, sizeof(i128)), *c_qH = calloc(MAX_C, sizeof(i128));
    for (int c = 0; c < MAX_C; c++) { c_gain[c] = -1.0; c_feat[c] = -1; }
    int ok = 0;
    for (int c = 0; c < MAX_C; c++) ok |= alloc_hist(&hs[c], mode, p, max_bins);
    if (ok) return -1;

    int root = node_count++;
    double Gr, Hr; i128 qGr, qHr;
    node_sums(&P, g, h, qg, qh, idx, 0, n_sub, &Gr, &Hr, &qGr, &qHr);
    double root_val = -Gr / (Hr + lam);
    int done = 0;
    if (n_sub < msl || Hr < mcw) {
        tf[root] = -1; tv[root] = root_val; done = 1;
    }
    if (!done) {
        build_hist(&P, &hs[0], max_bins, Xb, p, g, h, qg, qh, idx, 0, n_sub, fidx, nf, counts);
        split_t s = find_split(&P, &hs[0], max_bins, fidx, nf, counts, qGr, qHr);
        c_node[0] = root; c_start[0] = 0; c_end[0] = n_sub; c_depth[0] = 0;
        c_gain[0] = s.feat >= 0 ? s.gain : -1.0; c_feat[0] = s.feat; c_bin[0] = s.bin | (s.nr << 16);
        c_val[0] = root_val; c_active[0] = 1; c_qG[0] = qGr; c_qH[0] = qHr;
        if (s.feat < 0) { tf[root] = -1; tv[root] = root_val; done = 1; }
    }
    int n_splits = 0;
    while (!done && n_splits < max_leaves - 1) {
        int ci = -1; double bg = gamma;                    /* E:645-653 */
        for (int c = 0; c < MAX_C; c++)
            if (c_active[c] && c_feat[c] >= 0 && c_gain[c] > bg) { bg = c_gain[c]; ci = c; }
        if (ci < 0) break;
        int cur = c_node[ci];
        int64_t a = c_start[ci], b = c_end[ci];
        int depth = c_depth[ci];
        int64_t sp = partition(idx, a, b, Xb, p, c_feat[ci], c_bin[ci] & 0xffff, c_bin[ci] >> 16);
        int64_t nl = sp - a, nr = b - sp;
        if (nl < msl || nr < msl) {                          /* E:678-683 */
            tf[cur] = -1; tv[cur] = c_val[ci]; c_active[ci] = 0;
            continue;
        }
        int lid = node_count++, rid = node_count++;
        tf[cur] = c_feat[ci]; tt[cur] = (c_bin[ci] & 0xffff) | ((int64_t)(c_bin[ci] >> 16) << 32);
        tl[cur] = lid; tr[cur] = rid;
        tv[cur] = c_val[ci]; sg[cur] = c_gain[ci];
        n_splits++;
        int nd = depth + 1;
        int left_small = nl <= nr;
        int64_t sa = left_small ? a : sp, sb = left_small ? sp : b;
        int64_t la = left_small ? sp : a, lb = left_small ? b : sp;
        int sid = left_small ? lid : rid, gid = left_small ? rid : lid;
        int ss = -1, sl = -1;                                  /* E:712-720 */
        for (int c = 0; c < MAX_C; c++) {
            if (c != ci && !c_active[c]) {
                if (ss < 0) ss = c; else if (sl < 0) { sl = c; break; }
            }
        }
        build_hist(&P, &hs[ss], max_bins, Xb, p, g, h, qg, qh, idx, sa, sb, fidx, nf, counts);
        subtract_hist(&P, &hs[sl], &hs[ci], &hs[ss], max_bins, fidx, nf, counts);
        c_active[ci] = 0;
        for (int pass = 0; pass < 2; pass++) {
            int64_t ca = pass ? la : sa, cb = pass ? lb : sb;
            int cid = pass ? gid : sid, cs = pass ? sl : ss;
            double Gc, Hc; i128 qGc, qHc;
            node_sums(&P, g, h, qg, qh, idx, ca, cb, &Gc, &Hc, &qGc, &qHc);
            double val = -Gc / (Hc + lam);
            split_t s = { -1, 0, -1e9, 0 };
            int can = (cb - ca) >= msl && Hc >= mcw && nd < max_depth;
            if (can) s = find_split(&P, &hs[cs], max_bins, fidx, nf, counts, qGc, qHc);
            c_node[cs] = cid; c_start[cs] = ca; c_end[cs] = cb; c_depth[cs] = nd;
            c_gain[cs] = s.feat >= 0 ? s.gain : -1.0; c_feat[cs] = s.feat; c_bin[cs] = s.bin | (s.nr << 16);
            c_val[cs] = val; c_active[cs] = 1; c_qG[cs] = qGc; c_qH[cs] = qHc;
        }
    }
    if (!done)
        for (int c = 0; c < MAX_C; c++)
            if (c_active[c]) { tf[c_node[c]] = -1; tv[c_node[c]] = c_val[c]; }
    *n_nodes = node_count;
    for (int c = 0; c < MAX_C; c++) free_hist(&hs[c]);
    free(hs); free(c_node); free(c_depth); free(c_feat); free(c_bin); free(c_active);
    free(c_start); free(c_end); free(c_gain); free(c_val); free(c_qG); free(c_qH);
    free(idx); free(qg); free(qh);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Depth-wise (DFS) builder: E:233-508 (numeric features only).         */
/* ------------------------------------------------------------------ */
int or_build_depthwise(const uint16_t *Xb, int64_t n_all, int32_t p, const double *g,
                       const double *h, const int64_t *sample_idx, int64_t n_sub,
                       const int32_t *fidx, int32_t nf, const int32_t *counts,
                       int32_t max_bins, int32_t max_depth, int32_t msl, double mcw,
                       double lam, double gamma, int32_t mode, int32_t scale_bits,
                       int32_t *tf, int64_t *tt, double *tv, int32_t *tl, int32_t *tr,
                       double *sg, int32_t *n_nodes) {
    (void)gamma;  /* E:233-508 never reads gamma during growth */
    params_t P = { mode, scale_bits, lam, mcw, gamma, msl, max_depth, 0 };
    int max_nodes = (1 << (max_depth + 1)) - 1;
    for (int k = 0; k < max_nodes; k++) { tf[k] = -1; tt[k] = 0; tv[k] = 0.0; tl[k] = -1; tr[k] = -1; sg[k] = 0.0; }
    int node_count = 0;
    int64_t *idx = malloc(sizeof(int64_t) * (size_t)(n_sub > 0 ? n_sub : 1));
    memcpy(idx, sample_idx, sizeof(int64_t) * (size_t)n_sub);
    i128 *qg, *qh;
    quantize_all(&P, g, h, n_all, &qg, &qh);
    int SS = max_depth * 2 + 4;
    int32_t *s_node = calloc(SS, 4), *s_depth = calloc(SS, 4), *s_has = calloc(SS, 4);
    int64_t *s_a = calloc(SS, 8), *s_b = calloc(SS, 8);
    hist_t *sh = calloc((size_t)SS, sizeof(hist_t));
    hist_t work;
    for (int c = 0; c < SS; c++) alloc_hist(&sh[c], mode, p, max_bins);
    alloc_hist(&work, mode, p, max_bins);
    int sp_ = 0;
    s_node[0] = node_count++; s_a[0] = 0; s_b[0] = n_sub; s_depth[0] = 0; s_has[0] = 0; sp_ = 1;
    size_t cells = (size_t)p * max_bins;
    while (sp_ > 0) {
        sp_--;
        int cur = s_node[sp_]; int64_t a = s_a[sp_], b = s_b[sp_];
        int depth = s_depth[sp_], has = s_has[sp_], slot = sp_;
        double Gs, Hs; i128 qG, qH;
        node_sums(&P, g, h, qg, qh, idx, a, b, &Gs, &Hs, &qG, &qH);
        double val = -Gs / (Hs + lam);
        if (depth >= max_depth || (b - a) < msl || Hs < mcw) { tf[cur] = -1; tv[cur] = val; continue; }
        if (has) {
            for (int jj = 0; jj < nf; jj++) {
                int j = fidx[jj]; int64_t o = (int64_t)j * max_bins;
                for (int k = 0; k < counts[j]; k++) {
                    if (mode == OR_MODE_REF) { work.G[o + k] = sh[slot].G[o + k]; work.H[o + k] = sh[slot].H[o + k]; }
                    else { work.QG[o + k] = sh[slot].QG[o + k]; work.QH[o + k] = sh[slot].QH[o + k]; }
                }
            }
        } else {
            build_hist(&P, &work, max_bins, Xb, p, g, h, qg, qh, idx, a, b, fidx, nf, counts);
        }
        split_t s = find_split(&P, &work, max_bins, fidx, nf, counts, qG, qH);
        if (s.feat < 0) { tf[cur] = -1; tv[cur] = val; continue; }
        int64_t spos = partition(idx, a, b, Xb, p, s.feat, s.bin, s.nr);
        int64_t nl = spos - a, nr = b - spos;
        if (nl < msl || nr < msl) { tf[cur] = -1; tv[cur] = val; continue; }
        int lid = node_count++, rid = node_count++;
        tf[cur] = s.feat; tt[cur] = s.bin | ((int64_t)s.nr << 32); tl[cur] = lid; tr[cur] = rid; tv[cur] = val; sg[cur] = s.gain;
        int left_small = nl <= nr;
        int64_t sa = left_small ? a : spos, sb = left_small ? spos : b;
        int64_t la = left_small ? spos : a, lb = left_small ? b : spos;
        int sid = left_small ? lid : rid, gid = left_small ? rid : lid;
        int small_slot = sp_ + 1, large_slot = sp_;
        /* E:463-482: the smaller child's histogram is built row-major
         * (rows outer, features inner); per bin this is the same sequence
         * of additions as the feature-outer loop. */
        build_hist(&P, &sh[small_slot], max_bins, Xb, p, g, h, qg, qh, idx, sa, sb, fidx, nf, counts);
        subtract_hist(&P, &sh[large_slot], &work, &sh[small_slot], max_bins, fidx, nf, counts);
        (void)cells;
        s_node[sp_] = gid; s_a[sp_] = la; s_b[sp_] = lb; s_depth[sp_] = depth + 1; s_has[sp_] = 1; sp_++;
        s_node[sp_] = sid; s_a[sp_] = sa; s_b[sp_] = sb; s_depth[sp_] = depth + 1; s_has[sp_] = 1; sp_++;
    }
    *n_nodes = node_count;
    for (int c = 0; c < SS; c++) free_hist(&sh[c]);
    free_hist(&work); free(sh); free(s_node); free(s_depth); free(s_has); free(s_a); free(s_b);
    free(idx); free(qg); free(qh);
    return 0;
}

/* Bottom-up prune of both-leaf parents with gain < gamma (E:827-841). */
void or_post_prune(int32_t *tf, int32_t *tl, int32_t *tr, const double *sg, double gamma,
                   int32_t nc) {
    for (int k = nc - 1; k >= 0; k--) {
        if (tf[k] != -1) {
            int l = tl[k], r = tr[k];
            if (tf[l] == -1 && tf[r] == -1 && sg[k] < gamma) { tf[k] = -1; tl[k] = -1; tr[k] = -1; }
        }
    }
}

/* ------------------------------------------------------------------ */
/* Predict (E:843-884).                                                 */
/* ------------------------------------------------------------------ */
/* Leaf node id of every row for one tree (E:843-861 returns values[leaf]). */
void or_leaf_ids(const uint16_t *Xb, int64_t n, int32_t p, const int32_t *tf, const int64_t *tt,
                 const int32_t *tl, const int32_t *tr, int32_t *leaf) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int node = 0;
        while (tf[node] >= 0)
            node = goes_left(Xb[i * p + tf[node]], tt[node] & 0xffffffffLL, (int)(tt[node] >> 32)) ? tl[node] : tr[node];
        leaf[i] = node;
    }
}

/* F[i] = sum_t lr * values[leaf_t(i)] over a packed ensemble (E:863-884). */
void or_predict_packed(const uint16_t *Xb, int64_t n, int32_t p, const int16_t *feat,
                       const int64_t *thr, const double *val, const int32_t *left,
                       const int32_t *right, const int32_t *offsets, int32_t n_trees,
                       double lr, const uint8_t *nanr, double *F) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        double acc = 0.0;
        const uint16_t *row = Xb + i * p;
        for (int t = 0; t < n_trees; t++) {
            int o = offsets[t], node = 0;
            while (feat[o + node] >= 0) {
                node = goes_left(row[feat[o + node]], thr[o + node], nanr ? nanr[o + node] : 0) ? left[o + node]
                                                                                             : right[o + node];
            }
            acc += lr * val[o + node];
        }
        F[i] = acc;
    }
}

/* ------------------------------------------------------------------ */
/* Gradient / hessian / logloss (E:2861, E:2873-2874, E:2320-2325).     */
/* ------------------------------------------------------------------ */
void or_grad_hess(const double *F, const uint8_t *y, const double *w2, int64_t n,
                  double *g, double *h) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        double f = F[i];
        if (f < -500.0) f = -500.0; else if (f > 500.0) f = 500.0;
        double pr = 1.0 / (1.0 + exp(-f));
        double w = w2[y[i]];
        g[i] = w * (pr - (double)y[i]);
        h[i] = w * pr * (1.0 - pr);
    }
}

double or_logloss(const double *F, const uint8_t *y, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; i++) {
        double f = F[i];
        if (f < -500.0) f = -500.0; else if (f > 500.0) f = 500.0;
        double pr = 1.0 / (1.0 + exp(-f));
        if (pr < 1e-15) pr = 1e-15; else if (pr > 1.0 - 1e-15) pr = 1.0 - 1e-15;
        s += y[i] ? log(pr) : log(1.0 - pr);
    }
    return -s / (double)n;
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* (double)(hi * 2^64 + lo) -- exposes the oracle's int128 conversion. */
double or_i128_to_double(int64_t hi, uint64_t lo) {
    i128 v = ((i128)hi << 64) | (i128)lo;
    return i128_to_double(v);
}
