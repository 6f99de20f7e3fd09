// gbm_kernels.cuh -- the engine's CUDA kernels (sm_100a).
//
// Reference: src/bsscl_gbm/estimator_v1_0_1.py ("E").  Each kernel notes the
// reference lines whose computation it performs.
#pragma once

#include "gbm_common.cuh"

namespace gbm {

// ===========================================================================
// layout, gradients, F update
// ===========================================================================

// Row-major uint8 [rows][p] -> column blocks [nblk][n][16], ids clamped to
// bin_count-1 (E:593-594 clamps the same way; E:604 never splits above).
// A kernel launched with programmatic stream serialization may start while
// its predecessor drains; this waits until the predecessor has finished and
// its writes are visible (a no-op for a plain launch).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename T>
__global__ void k_pack_bins(const T *__restrict__ src, int64_t rows, int p, int64_t row0,
                            int64_t n, int nblk, const int32_t *__restrict__ counts,
                            uint8_t *__restrict__ xb) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows * nblk) return;
    int64_t r = t / nblk;
    int b = (int)(t % nblk);
    uint8_t v[16];
#pragma unroll
    for (int k = 0; k < 16; k++) {
        int f = b * kBlk + k;
        uint8_t x = 0;
        if (f < p) {
            int c = src[r * p + f];
            int lim = min(counts[f] - 1, 255);   // a 257-bin feature's id 256 is kept in its top bits
            x = (uint8_t)(c > lim ? lim : c);
        }
        v[k] = x;
    }
    uint4 o;
    memcpy(&o, v, 16);
    reinterpret_cast<uint4 *>(xb)[(int64_t)b * n + row0 + r] = o;
}


// F = base score for every row (E:2837), and the first round's quantised (g, h).
__global__ void k_init_grad(double *__restrict__ F, const uint8_t *__restrict__ y, int64_t n, double base,
                            double w0, double w1, double scale, longlong2 *__restrict__ q) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    F[i] = base;
    int yi = y[i];
    double g, h, p;
    grad_hess(base, yi, yi ? w1 : w0, g, h, p);
    q[i] = make_longlong2(__double2ll_rn(__dmul_rn(g, scale)), __double2ll_rn(__dmul_rn(h, scale)));
}

__global__ void k_quant(const double *__restrict__ g, const double *__restrict__ h, int64_t n, double scale,
                        longlong2 *__restrict__ q) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    q[i] = make_longlong2(__double2ll_rn(__dmul_rn(g[i], scale)), __double2ll_rn(__dmul_rn(h[i], scale)));
}

__global__ void k_export_grad(const double *__restrict__ F, const uint8_t *__restrict__ y, int64_t n,
                              double w0, double w1, double *__restrict__ g, double *__restrict__ h) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int yi = y[i];
    double gg, hh, p;
    grad_hess(F[i], yi, yi ? w1 : w0, gg, hh, p);
    g[i] = gg;
    h[i] = hh;
}

// One pass over all rows: traverse the round's tree (E:843-861), F += lr * v
// with two separately rounded operations like NumPy's F += lr * pred
// (E:2896-2897), the logloss term of the updated F (E:2905) and the next
// round's quantised (g, h) (E:2861, E:2873-2874).
__global__ void __launch_bounds__(kUpdThreads)
k_update(const TreeDev *__restrict__ tree, const uint8_t *__restrict__ xb, int64_t n,
         const uint8_t *__restrict__ y, double w0, double w1, double lr, double scale,
         double *__restrict__ F, longlong2 *__restrict__ q, int32_t *__restrict__ leaf_out,
         double *__restrict__ loss_part, unsigned *__restrict__ done, double *__restrict__ loss_out,
         const int32_t *__restrict__ bigidx, const uint32_t *__restrict__ topbits) {
    griddep_wait();
    __shared__ int s_feat[256], s_thr[256], s_left[256], s_right[256];
    __shared__ double s_val[256];
    __shared__ double s_red[kUpdThreads / 32];
    int nn = tree->n;
    if (nn <= 0) return;   // the replay failed; the host reports it and F is left as it was
    for (int k = threadIdx.x; k < nn; k += blockDim.x) {
        s_feat[k] = tree->feat[k];
        s_thr[k] = tree->thr[k];
        s_left[k] = tree->left[k];
        s_right[k] = tree->right[k];
        s_val[k] = tree->val[k];
    }
    __syncthreads();
    double acc = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int node = 0;
        while (s_feat[node] >= 0) {
            int b = bin_of(xb, n, i, s_feat[node]);
            const int th = s_thr[node] & 0xffff;
            node = goes_left(b, th, s_thr[node] >> 16) &&
                           !(th >= 255 && top_bit(topbits, (n + 31) >> 5, bigidx[s_feat[node]], i))
                       ? s_left[node] : s_right[node];
        }
        if (leaf_out) leaf_out[i] = node;
        double f = __dadd_rn(F[i], __dmul_rn(lr, s_val[node]));
        F[i] = f;
        int yi = y[i];
        double g, h, p;
        grad_hess(f, yi, yi ? w1 : w0, g, h, p);
        acc += loss_term(p, yi);
        q[i] = make_longlong2(__double2ll_rn(__dmul_rn(g, scale)), __double2ll_rn(__dmul_rn(h, scale)));
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < kUpdThreads / 32; w++) s += s_red[w];
        loss_part[blockIdx.x] = s;
    }
    // the last block sums the partials (k_sum_partials' fixed order: thread t
    // takes blocks t, t+256, ..., then thread 0 adds the 256 sums in order)
    __shared__ int s_last;
    __shared__ double s_sum[kUpdThreads];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    double a = 0.0;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) a += __ldcg(loss_part + b);
    s_sum[threadIdx.x] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
        *done = 0;
        double t = 0.0;
        for (int k = 0; k < (int)blockDim.x; k++) t += s_sum[k];
        *loss_out = t;
    }
}

// ---------------------------------------------------------------------------
// multi-class softmax (E:2949-3065): K trees per round on one shared sample
// ---------------------------------------------------------------------------

// NumPy's sum of a short contiguous row (pairwise_sum for n <= 128: a plain
// loop from 0 below 8 terms, else 8 running sums combined pairwise, then the
// remainder) -- the order of exp_F.sum(axis=1) in _softmax (E:2331).
__device__ __forceinline__ double np_row_sum(const double *a, int n) {
    if (n < 8) {
        double r = 0.0;
        for (int i = 0; i < n; i++) r = __dadd_rn(r, a[i]);
        return r;
    }
    double r[8];
#pragma unroll
    for (int j = 0; j < 8; j++) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
#pragma unroll
        for (int j = 0; j < 8; j++) r[j] = __dadd_rn(r[j], a[i + j]);
    double res = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                           __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
    for (; i < n; i++) res = __dadd_rn(res, a[i]);
    return res;
}

constexpr int kMaxClasses = 64;

// Per row: p = softmax(F[:, i]) (E:2328-2332), then for every class k
// g = w_y (p_k - [y == k]), h = max(w_y p_k (1 - p_k), 1e-8) (E:2991-2992,
// E:2997), quantised to the 2^-S grid; and the row's logloss term
// log(clip(p_y, 1e-15, 1 - 1e-15)) (E:2335-2341).  F and q are class-major
// ([k][n]).
__global__ void __launch_bounds__(kUpdThreads)
k_softmax_grad(const double *__restrict__ F, const uint8_t *__restrict__ y, int64_t n, int K,
               const double *__restrict__ w, double scale, longlong2 *__restrict__ q,
               double *__restrict__ loss_part) {
    griddep_wait();
    __shared__ double s_red[kUpdThreads / 32];
    double acc = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        double e[kMaxClasses];
        double m = F[i];
        for (int k = 1; k < K; k++) m = fmax(m, F[(int64_t)k * n + i]);
        for (int k = 0; k < K; k++) e[k] = exp(__dsub_rn(F[(int64_t)k * n + i], m));
        const double s = np_row_sum(e, K);
        const int yi = y[i];
        const double wi = w[yi];
        for (int k = 0; k < K; k++) {
            const double pk = __ddiv_rn(e[k], s);
            const double g = __dmul_rn(wi, __dsub_rn(pk, k == yi ? 1.0 : 0.0));
            const double h = fmax(__dmul_rn(__dmul_rn(wi, pk), __dsub_rn(1.0, pk)), 1e-8);
            q[(int64_t)k * n + i] = make_longlong2(__double2ll_rn(__dmul_rn(g, scale)), __double2ll_rn(__dmul_rn(h, scale)));
            if (k == yi) acc += log(fmin(fmax(pk, 1e-15), 1.0 - 1e-15));
        }
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w2 = 0; w2 < kUpdThreads / 32; w2++) s += s_red[w2];
        loss_part[blockIdx.x] = s;
    }
}

// F_k += lr * value(leaf) for one class's tree (E:3001-3002); the gradients
// of the next round come from k_softmax_grad once all K trees are in.
__global__ void __launch_bounds__(kUpdThreads)
k_update_class(const TreeDev *__restrict__ tree, const uint8_t *__restrict__ xb, int64_t n, double lr,
               double *__restrict__ F, int32_t *__restrict__ leaf_out, const int32_t *__restrict__ bigidx,
               const uint32_t *__restrict__ topbits) {
    griddep_wait();
    __shared__ int s_feat[256], s_thr[256], s_left[256], s_right[256];
    __shared__ double s_val[256];
    const int nn = tree->n;
    if (nn <= 0) return;
    for (int k = threadIdx.x; k < nn; k += blockDim.x) {
        s_feat[k] = tree->feat[k];
        s_thr[k] = tree->thr[k];
        s_left[k] = tree->left[k];
        s_right[k] = tree->right[k];
        s_val[k] = tree->val[k];
    }
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int node = 0;
        while (s_feat[node] >= 0) {
            const int b = bin_of(xb, n, i, s_feat[node]);
            const int th = s_thr[node] & 0xffff;
            node = goes_left(b, th, s_thr[node] >> 16) &&
                           !(th >= 255 && top_bit(topbits, (n + 31) >> 5, bigidx[s_feat[node]], i))
                       ? s_left[node] : s_right[node];
        }
        if (leaf_out) leaf_out[i] = node;
        F[i] = __dadd_rn(F[i], __dmul_rn(lr, s_val[node]));
    }
}

// ---------------------------------------------------------------------------
// regression (E:2607-2705): g = F - y (mse) or sign(F - y) (mae), h = 1
// ---------------------------------------------------------------------------

__device__ __forceinline__ double reg_grad(double f, double y, int mae) {
    const double d = __dsub_rn(f, y);
    if (!mae) return d;
    return d > 0.0 ? 1.0 : (d < 0.0 ? -1.0 : 0.0);   // np.sign
}

// F = init score (E:2613-2614).
__global__ void k_fill(double *__restrict__ F, int64_t n, double v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) F[i] = v;
}

// The round's quantised gradients on the grid 2^-S.
__global__ void k_reg_quant(const double *__restrict__ F, const double *__restrict__ y, int64_t n, int mae,
                            double scale, longlong2 *__restrict__ q) {
    griddep_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    q[i] = make_longlong2(__double2ll_rn(__dmul_rn(reg_grad(F[i], y[i], mae), scale)), __double2ll_rn(scale));
}

// F += lr * value(leaf) (E:2660-2661); per block the loss partial
// sum (y - F)^2 or |y - F| (E:2663) and the largest |g| of the next round.
__global__ void __launch_bounds__(kUpdThreads)
k_update_reg(const TreeDev *__restrict__ tree, const uint8_t *__restrict__ xb, int64_t n, double lr,
             double *__restrict__ F, const double *__restrict__ y, int mae, int32_t *__restrict__ leaf_out,
             double *__restrict__ loss_part, double *__restrict__ gmax_part, const int32_t *__restrict__ bigidx,
             const uint32_t *__restrict__ topbits) {
    griddep_wait();
    __shared__ int s_feat[256], s_thr[256], s_left[256], s_right[256];
    __shared__ double s_val[256];
    __shared__ double s_red[kUpdThreads / 32], s_mx[kUpdThreads / 32];
    const int nn = tree->n;
    if (nn <= 0) return;
    for (int k = threadIdx.x; k < nn; k += blockDim.x) {
        s_feat[k] = tree->feat[k];
        s_thr[k] = tree->thr[k];
        s_left[k] = tree->left[k];
        s_right[k] = tree->right[k];
        s_val[k] = tree->val[k];
    }
    __syncthreads();
    double acc = 0.0, mx = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int node = 0;
        while (s_feat[node] >= 0) {
            const int b = bin_of(xb, n, i, s_feat[node]);
            const int th = s_thr[node] & 0xffff;
            node = goes_left(b, th, s_thr[node] >> 16) &&
                           !(th >= 255 && top_bit(topbits, (n + 31) >> 5, bigidx[s_feat[node]], i))
                       ? s_left[node] : s_right[node];
        }
        if (leaf_out) leaf_out[i] = node;
        const double f = __dadd_rn(F[i], __dmul_rn(lr, s_val[node]));
        F[i] = f;
        const double r = __dsub_rn(y[i], f);
        acc += mae ? fabs(r) : __dmul_rn(r, r);
        mx = fmax(mx, fabs(reg_grad(f, y[i], mae)));
    }
    acc = warp_sum(acc);
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_down_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) {
        s_red[threadIdx.x >> 5] = acc;
        s_mx[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0, m = 0.0;
        for (int w2 = 0; w2 < kUpdThreads / 32; w2++) {
            s += s_red[w2];
            m = fmax(m, s_mx[w2]);
        }
        loss_part[blockIdx.x] = s;
        gmax_part[blockIdx.x] = m;
    }
}

// max of the per-block partials (one thread; a few hundred values)
__global__ void k_max_partials(const double *__restrict__ part, int m, double *__restrict__ out) {
    griddep_wait();
    if (threadIdx.x || blockIdx.x) return;
    double v = 0.0;
    for (int k = 0; k < m; k++) v = fmax(v, part[k]);
    *out = v;
}

// The quantised (g, h) of n rows as float64 (exact: |q| < 2^53).
__global__ void k_export_q(const longlong2 *__restrict__ q, int64_t n, double inv_scale, double *__restrict__ g,
                           double *__restrict__ h) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const longlong2 v = q[i];
    g[i] = __dmul_rn((double)v.x, inv_scale);
    h[i] = __dmul_rn((double)v.y, inv_scale);
}

// Fixed-order sum of the per-block loss partials (deterministic).
__global__ void k_sum_partials(const double *__restrict__ part, int m, double *__restrict__ out) {
    griddep_wait();
    __shared__ double s[256];
    double a = 0.0;
    for (int k = threadIdx.x; k < m; k += blockDim.x) a += part[k];
    s[threadIdx.x] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < (int)blockDim.x; k++) t += s[k];
        *out = t;
    }
}

// ===========================================================================
// in-bag compaction: mask -> ascending row ids
// ===========================================================================

// (the mask's compaction into row ids, k_compact_rows, uses the partition's look-back below)

// In-bag mask of this rank's rows [row0, row0 + n) from global row ids.
__global__ void k_mask_from_rows(const int32_t *__restrict__ rows, int64_t m, int64_t row0, int64_t n,
                                 uint8_t *__restrict__ mask) {
    griddep_wait();
    int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= m) return;
    int64_t r = (int64_t)rows[k] - row0;
    if (r >= 0 && r < n) mask[r] = 1;
}

// ---------------------------------------------------------------------------
// The round's row shuffle from its swap targets (the sampler's NumPy legacy
// Fisher-Yates, E:2502-2517), in parallel.  Steps run i = n-1 .. 1 and step
// i swaps positions i and j_i <= i; position i is final after step i.  With
//   m(q)  = min{ i > q : j_i = q }          (the last write into q before step q)
//   mp(i) = min{ i' > i : j_i' = j_i }     (the last write into j_i before step i)
//   P(i)  = value at position i just before step i = P(m(i)), or i if m(i) = none
// the round's permutation of arange(n) is S[i] = P(mp(i)) or j_i, and
// S[0] = P(m(0)) or 0.  m only increases along a chain, so every chase ends.
// The targets arrive forward: t[k] = j_(n-1-k).
// ---------------------------------------------------------------------------

// Bucket the steps by target: a singly linked list per position.
__global__ void k_shuf_link(const int32_t *__restrict__ t, int64_t n, int32_t *__restrict__ head,
                            int32_t *__restrict__ nxt) {
    griddep_wait();
    int64_t i = 1 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int q = t[n - 1 - i];
    nxt[i] = atomicExch(&head[q], (int32_t)i);
}

__device__ __forceinline__ int32_t min_above(const int32_t *__restrict__ head, const int32_t *__restrict__ nxt,
                                             int q, int64_t floor_) {
    int32_t best = -1;
    for (int32_t e = head[q]; e >= 0; e = nxt[e])
        if (e > floor_ && (best < 0 || e < best)) best = e;
    return best;
}

__global__ void k_shuf_min(const int32_t *__restrict__ t, int64_t n, const int32_t *__restrict__ head,
                           const int32_t *__restrict__ nxt, int32_t *__restrict__ m, int32_t *__restrict__ mp) {
    griddep_wait();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    m[i] = min_above(head, nxt, (int)i, i);
    if (i >= 1) mp[i] = min_above(head, nxt, t[n - 1 - i], i);
}

// perm_out = perm_in[S] (the shuffle applied to the cumulative permutation).
__global__ void k_shuf_compose(const int32_t *__restrict__ t, int64_t n, const int32_t *__restrict__ m,
                               const int32_t *__restrict__ mp, const int32_t *__restrict__ perm_in,
                               int32_t *__restrict__ perm_out) {
    griddep_wait();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int32_t src = i == 0 ? m[0] : mp[i];
    int32_t s;
    if (src < 0) {
        s = i == 0 ? 0 : t[n - 1 - i];
    } else {
        int32_t r = src;
        for (int32_t nx = m[r]; nx >= 0; nx = m[nx]) r = nx;
        s = r;
    }
    perm_out[i] = perm_in[s];
}

// Throughput-mode in-bag mask of this rank's rows (gbm_row_hash).
__global__ void k_mask_hash(uint8_t *__restrict__ mask, int64_t n, int64_t row0, uint64_t seed, uint64_t thr,
                            const long long *__restrict__ round_p) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t r = (uint64_t)*round_p;
    mask[i] = thr == ~0ull ? 1 : (gbm_row_hash(seed, r, (uint64_t)(row0 + i)) < thr ? 1 : 0);
}

__global__ void k_iota(int32_t *__restrict__ a, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = (int32_t)i;
}


// ===========================================================================
// the top bin of 257-bin features
// ===========================================================================

// Top bits from a list of (row, big feature index) pairs (the uint16 upload,
// whose ids the host narrows to uint8).
__global__ void k_set_topbits(const int64_t *__restrict__ pairs, int64_t m, int64_t words_per,
                              uint32_t *__restrict__ bits) {
    griddep_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const int64_t r = pairs[2 * i], b = pairs[2 * i + 1];
    atomicOr(bits + b * words_per + (r >> 5), 1u << (r & 31));
}

// Rows with a top bit, per big feature (one CTA each), in ascending order:
// cnt[b] first (count pass), then rows[off[b] ..] (fill pass).
template <bool FILL>
__global__ void __launch_bounds__(256) k_top_list(const uint32_t *__restrict__ bits, int64_t words_per, int64_t n,
                                                  int32_t *__restrict__ cnt, const int32_t *__restrict__ off,
                                                  int32_t *__restrict__ rows) {
    griddep_wait();
    __shared__ int s_w[8];
    const int b = blockIdx.x;
    const uint32_t *w = bits + (int64_t)b * words_per;
    int carry = 0;
    for (int64_t w0 = 0; w0 < words_per; w0 += 256) {
        const int64_t wi = w0 + threadIdx.x;
        uint32_t x = wi < words_per ? w[wi] : 0u;
        int tot;
        const int e = block_excl_scan(__popc(x), s_w, tot);
        if (FILL) {
            int o = off[b] + carry + e;
            while (x) {
                const int k = __ffs(x) - 1;
                x &= x - 1;
                const int64_t r = wi * 32 + k;
                if (r < n) rows[o++] = (int32_t)r;
            }
        }
        carry += tot;
    }
    if (!FILL && threadIdx.x == 0) cnt[b] = carry;
}

// The top cells of a level's histograms: one CTA per big feature b; for
// every histogram task t of the level (when the round selected b, at
// position jj) each row of b's top list that lies in the task's row
// segment (ascending or descending: k_partition keeps every node's list
// monotonic, so a binary search) adds its (g, h) into the task's staging
// top cell jj, as (hi, lo) words like the cells.  Top rows are the
// rows equal to the column maximum: few, against the segment's length.
__global__ void __launch_bounds__(128) k_hist_top(const int32_t *__restrict__ rows0, const int32_t *__restrict__ rows1,
                                                  const HistTask *__restrict__ tasks, const int *__restrict__ ntask_p,
                                                  const int32_t *__restrict__ bigfeat, const int16_t *__restrict__ fpos,
                                                  const int32_t *__restrict__ top_off,
                                                  const int32_t *__restrict__ top_rows, int nf,
                                                  const longlong2 *__restrict__ q, long long *__restrict__ stage_hist,
                                                  const unsigned long long *__restrict__ par_word, int64_t par_stride) {
    griddep_wait();
    if (par_word) stage_hist += (int64_t)(*par_word & 1ull) * par_stride;
    const int b = blockIdx.x;
    const int jj = fpos[bigfeat[b]];
    if (jj < 0) return;
    const int ntask = *ntask_p, i0 = top_off[b], i1 = top_off[b + 1];
    for (int t = 0; t < ntask; t++) {
        const HistTask tk = tasks[t];
        const int32_t *rows = tk.buf ? rows1 : rows0;
        long long *cellp = stage_hist + (int64_t)tk.stage * slot_words_for(nf) + top_cell_offset(nf, jj);
        if (tk.end <= tk.begin) continue;
        const bool asc = rows[tk.begin] <= rows[tk.end - 1];
        for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
            const int r = top_rows[i];
            long long lo = tk.begin, hi = tk.end;   // the first position at or past r in the list's order
            while (lo < hi) {
                const long long mid = (lo + hi) >> 1;
                if (asc ? rows[mid] < r : rows[mid] > r) lo = mid + 1; else hi = mid;
            }
            if (lo < tk.end && rows[lo] == r) {
                const longlong2 qq = q[r];
                atomicAdd((unsigned long long *)(cellp + 0), (unsigned long long)(qq.x >> 32));
                atomicAdd((unsigned long long *)(cellp + 1), (unsigned long long)(qq.x & 0xffffffffll));
                atomicAdd((unsigned long long *)(cellp + 2), (unsigned long long)(qq.y >> 32));
                atomicAdd((unsigned long long *)(cellp + 3), (unsigned long long)(qq.y & 0xffffffffll));
            }
        }
    }
}

// ===========================================================================
// histograms
// ===========================================================================

__device__ __forceinline__ long long cost_bound(long long c, long long T, long long G) { return c * T / G; }
__device__ __forceinline__ long long ceil_div_ll(long long a, long long b) { return (a + b - 1) / b; }

// v rotated by r bytes (0 <= r < 16): byte k of the result is byte
// (k + r) mod 16 of v (bytes little-endian, word k / 4).
__device__ __forceinline__ uint4 rot_bytes(uint4 v, int r) {
    unsigned a = v.x, b = v.y, c = v.z, d = v.w;
    if (r & 8) {
        unsigned t0 = a, t1 = b;
        a = c; b = d; c = t0; d = t1;
    }
    if (r & 4) {
        unsigned t = a;
        a = b; b = c; c = d; d = t;
    }
    const unsigned sh = (unsigned)(r & 3) * 8u;
    return make_uint4(__funnelshift_r(a, b, sh), __funnelshift_r(b, c, sh), __funnelshift_r(c, d, sh),
                      __funnelshift_r(d, a, sh));
}

__device__ __forceinline__ unsigned byte_of(const uint4 &v, int k) {
    const unsigned w = (k >> 2) == 0 ? v.x : (k >> 2) == 1 ? v.y : (k >> 2) == 2 ? v.z : v.w;
    return (w >> ((k & 3) * 8)) & 0xffu;
}

// The round's selected features, packed into dense blocks of 16: block v,
// slot s holds the bin of feature fidx[16 v + s] (0 past the last one), in
// the same column-block layout as the bins themselves ([nvb][n][16]).  The
// histogram then runs 16 busy lanes per block: 70 selected features of 100
// take 5 blocks instead of 7 partly idle ones.  A CTA takes 256 rows: their
// records of every physical block are staged in shared memory at a 20-byte
// row stride (5 words, so 32 consecutive rows fall in 32 banks), then each
// thread assembles its row's packed records.
constexpr int kCompactRows = 256;
constexpr int kCompactStrideW = 5;   // words per staged record (16 bytes + pad)

__global__ void __launch_bounds__(kCompactRows)
k_compact_feat(const uint8_t *__restrict__ xb, int64_t n, int nblk, const int32_t *__restrict__ fidx, int nf,
               uint8_t *__restrict__ xc) {
    griddep_wait();
    extern __shared__ uint32_t cst[];   // [nblk][256][5] words, then fidx [nf]
    int32_t *s_f = reinterpret_cast<int32_t *>(cst + (size_t)nblk * kCompactRows * kCompactStrideW);
    const int64_t r0 = (int64_t)blockIdx.x * kCompactRows;
    const int t = threadIdx.x;
    const int64_t row = r0 + t;
    for (int i = t; i < nf; i += kCompactRows) s_f[i] = fidx[i];
    if (row < n) {
        for (int b = 0; b < nblk; b++) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(xb) + (int64_t)b * n + row);
            uint32_t *d = cst + ((size_t)b * kCompactRows + t) * kCompactStrideW;
            d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
        }
    }
    __syncthreads();
    if (row >= n) return;
    const uint8_t *sb = reinterpret_cast<const uint8_t *>(cst);
    const int nvb = (nf + kBlk - 1) / kBlk;
    for (int v = 0; v < nvb; v++) {
        uint32_t w[4];
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) {
            uint32_t x = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int pos = v * kBlk + q4 * 4 + k;
                if (pos < nf) {
                    const int f = s_f[pos];
                    x |= (uint32_t)sb[(((size_t)(f >> 4) * kCompactRows + t) * kCompactStrideW) * 4 + (f & 15)] << (8 * k);
                }
            }
            w[q4] = x;
        }
        reinterpret_cast<uint4 *>(xc)[(int64_t)v * n + row] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// k_hist3: the per-node gradient/hessian histograms of a level (the root,
// E:582-596, then the smaller child of every split, E:723-737), exact.
// * Fixed point: every row's (g, h) is a pair of int64 q values on the grid
//   2^-S.  Each q is split into three digits, q = top * 2^34 + mid * 2^17 +
//   low (low, mid in [0, 2^17), top signed), and each digit is summed in its
//   own 32-bit shared-memory word: native 32-bit shared atomics, six per
//   (row, feature), exact.
// * Layout: the lanes of a warp each load their own row's 16-byte record of
//   16 features; in step k lane l = 16 h + f adds feature (f + k) mod 16,
//   and half-warp h keeps its own copy of every cell: cell (digit d, bin b,
//   half h, feature f) is word ((d * 257 + b) * 2 + h) * 16 + f, whose bank
//   is 16 h + f.  The 32 lanes of an atomic instruction hit 32 different
//   banks whatever their bins: one wavefront per instruction.
// * Every bin is added, the NaN bin included, so no lane idles on it.
// * A slot whose feature the round did not select adds into a trash bin
//   (256): its cell sits in the lane's own bank like every other cell, so
//   the instruction stays conflict-free, and the trash row is never read.
// * Runs of up to kChunk3 = 32768 rows between flushes: (2^17 - 1) * 2^15 <
//   2^32 keeps the low and middle digit sums inside 32 bits, and the top
//   digit's |sum| < 2^14 * 2^15.  At the flush a cell's 128-bit value is
//   split into its words without forming it in 64 bits: with a = mid * 2^17
//   + low (< 2^50), hi = 4 * top + (a >> 32) and lo = a mod 2^32.  The
//   staging slot sums these (hi, lo) words over the CTAs of a segment (and
//   over ranks): value = hi * 2^32 + lo, exact.
constexpr int kHistV3Threads = 1024;
constexpr int kChunk3 = 32768;
constexpr int kBinsV3 = kBins + 1;                   // + the trash bin
constexpr int kDigV3 = kBinsV3 * 2 * kBlk;           // words between two digits
constexpr int kAccV3Words = 6 * kDigV3;              // 197,376 bytes

// COMPACT: xb is the round's packed blocks (k_compact_feat): block bi holds
// feature positions 16 bi .. 16 bi + 15, every slot below nf selected; the
// physical block list and feature positions are not read.
template <bool COMPACT>
__global__ void __launch_bounds__(kHistV3Threads, 1)
k_hist3(const uint8_t *__restrict__ xb, int64_t n, const int32_t *__restrict__ rows0,
        const int32_t *__restrict__ rows1, const HistTask *__restrict__ tasks, const int32_t *__restrict__ rpre,
        const int *__restrict__ ntask_p, const int32_t *__restrict__ blist, const int32_t *__restrict__ nb_p,
        const int16_t *__restrict__ fpos, int nf, const longlong2 *__restrict__ q, long long *__restrict__ stage_hist,
        const unsigned long long *__restrict__ par_word, int64_t par_stride, int seg_cost) {
    griddep_wait();
    if (par_word) stage_hist += (int64_t)(*par_word & 1ull) * par_stride;   // peer exchange: this level's buffer
    extern __shared__ unsigned acc[];   // [6][257][2][16]
    __shared__ long long s_tot[2][kHistV3Threads / 32];
    const int ntask = *ntask_p;
    const int nb = COMPACT ? (nf + kBlk - 1) / kBlk : *nb_p;
    if (ntask <= 0 || nb <= 0) return;
    // The work split.  Within a block, task t costs w per row plus seg_cost
    // for its segment (zeroing the accumulators and the flush, whatever its
    // rows): task t spans [w rpre[t] + C t, w rpre[t+1] + C (t+1)) of the
    // block's Wb = w R + C ntask, its rows after its first C units.  CTA c
    // takes [c T / G, (c+1) T / G) of T = nb Wb, so a CTA whose share covers
    // many small tasks takes fewer rows.
    const long long R = rpre[ntask];
    const long long w = kRowWeight, C = seg_cost;
    const long long Wb = w * R + C * ntask;
    const long long T = (long long)nb * Wb;
    if (T <= 0) return;
    const long long G = gridDim.x;
    const long long B0 = cost_bound(blockIdx.x, T, G), B1 = cost_bound(blockIdx.x + 1, T, G);
    if (B0 >= B1) return;
    // the first row at or after cost position y (0 <= y <= Wb) of a block
    auto row_at = [&](long long y) -> int {
        int lo = 0, hi = ntask;   // the last task t with w rpre[t] + C t <= y (t = ntask: past the end)
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (w * rpre[mid] + C * mid <= y) lo = mid; else hi = mid - 1;
        }
        if (lo >= ntask) return (int)R;
        const long long off = y - (w * rpre[lo] + C * lo) - C;
        const long long kk = off <= 0 ? 0 : ceil_div_ll(off, w);
        return (int)min((long long)rpre[lo + 1], rpre[lo] + kk);
    };
    const int lane = threadIdx.x & 31, half = lane >> 4, fl = lane & 15;
    const int warp = threadIdx.x >> 5;
    const int64_t slot_words = slot_words_for(nf);
    int bi = (int)min((long long)nb - 1, B0 / Wb);
    for (; bi < nb; bi++) {
        const long long base = Wb * bi;
        if (base >= B1) break;
        const int k0 = row_at(max(B0 - base, 0ll));
        const int k1 = row_at(min(B1 - base, Wb));
        if (k0 >= k1) continue;
        const int blk = COMPACT ? bi : blist[bi];
        unsigned mask = 0;
        if (COMPACT) {
            const int m = min(nf - bi * kBlk, kBlk);
            mask = m >= kBlk ? 0xffffu : (1u << m) - 1u;
        } else {
#pragma unroll
            for (int k = 0; k < kBlk; k++) mask |= (fpos[blk * kBlk + k] >= 0 ? 1u : 0u) << k;
        }
        // bit k set: step k's feature (fl + k) mod 16 is not selected -> trash bin
        const unsigned unsel = ~((mask | (mask << kBlk)) >> fl) & 0xffffu;
        const uint4 *xv = reinterpret_cast<const uint4 *>(xb) + (int64_t)blk * n;
        int t;
        {
            int lo = 0, hi = ntask - 1;
            while (lo < hi) {
                int mid = (lo + hi + 1) >> 1;
                if (rpre[mid] <= k0) lo = mid; else hi = mid - 1;
            }
            t = lo;
        }
        for (int k = k0; k < k1; t++) {
            const int t0 = rpre[t], t1 = rpre[t + 1];
            if (t1 <= k) continue;
            const HistTask tk = tasks[t];
            const int32_t *__restrict__ rows = tk.buf ? rows1 : rows0;
            const int pe = min(k1, t1);
            const bool single = k == t0 && pe == t1 && (t1 - t0) <= kChunk3;
            long long *dst = stage_hist + (int64_t)tk.stage * slot_words;
            for (int c0 = k; c0 < pe; c0 += kChunk3) {
                const int c1 = min(pe, c0 + kChunk3);
                for (int i = threadIdx.x; i < kAccV3Words / 4; i += blockDim.x)
                    reinterpret_cast<uint4 *>(acc)[i] = make_uint4(0u, 0u, 0u, 0u);
                __syncthreads();
                const int r0 = (int)tk.begin + (c0 - t0), r1 = (int)tk.begin + (c1 - t0);
                long long tg = 0, th = 0;
                unsigned *my = acc + half * kBlk;
                int rb = r0 + (int)(threadIdx.x & ~31u);
                int row_next = rb + lane < r1 ? rows[rb + lane] : 0;
                longlong2 q_next = rb + lane < r1 ? __ldg(q + row_next) : make_longlong2(0, 0);
                for (; rb < r1; rb += blockDim.x) {
                    const int r = rb + lane;
                    const bool valid = r < r1;
                    const int row = row_next;
                    const longlong2 qq = q_next;
                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                    if (valid) v = __ldg(xv + row);
                    // the next step's row id and q, in flight with this step's atomics
                    const bool vn = r + (int)blockDim.x < r1;
                    row_next = vn ? rows[r + blockDim.x] : 0;
                    q_next = vn ? __ldg(q + row_next) : make_longlong2(0, 0);
                    tg += qq.x;
                    th += qq.y;
                    // an invalid lane adds zeros (its q is 0) into real cells: harmless
                    const unsigned dg0 = (unsigned)qq.x & 0x1ffffu, dg1 = (unsigned)(qq.x >> kDig) & 0x1ffffu,
                                   dg2 = (unsigned)(int)(qq.x >> (2 * kDig));
                    const unsigned dh0 = (unsigned)qq.y & 0x1ffffu, dh1 = (unsigned)(qq.y >> kDig) & 0x1ffffu,
                                   dh2 = (unsigned)(int)(qq.y >> (2 * kDig));
                    const uint4 vr = rot_bytes(v, fl);
#pragma unroll
                    for (int k = 0; k < kBlk; k++) {
                        const unsigned b = ((unsel >> k) & 1u) ? (unsigned)kBins : byte_of(vr, k);
                        unsigned *cc = my + b * (2 * kBlk) + ((fl + k) & (kBlk - 1));
                        atomicAdd(cc + 0 * kDigV3, dg0);
                        atomicAdd(cc + 1 * kDigV3, dg1);
                        atomicAdd(cc + 2 * kDigV3, dg2);
                        atomicAdd(cc + 3 * kDigV3, dh0);
                        atomicAdd(cc + 4 * kDigV3, dh1);
                        atomicAdd(cc + 5 * kDigV3, dh2);
                    }
                }
                if (bi == 0) {
                    tg = warp_sum(tg);   // <= 32 rows per lane, 1024 per warp: |sum| < 2^58
                    th = warp_sum(th);
                    if (lane == 0) {
                        s_tot[0][warp] = tg;
                        s_tot[1][warp] = th;
                    }
                }
                __syncthreads();
                if (bi == 0 && threadIdx.x < 2) {
                    i128 tot = 0;
                    for (int w2 = 0; w2 < kHistV3Threads / 32; w2++) tot += (i128)s_tot[threadIdx.x][w2];
                    const long long thi = (long long)(tot >> 32), tlo = (long long)(tot & 0xffffffff);
                    long long *o = dst + (int64_t)nf * kBins * kWords + 2 * threadIdx.x;
                    if (single) {
                        o[0] = thi;
                        o[1] = tlo;
                    } else {
                        if (thi) atomicAdd((unsigned long long *)(o + 0), (unsigned long long)thi);
                        if (tlo) atomicAdd((unsigned long long *)(o + 1), (unsigned long long)tlo);
                    }
                }
                // flush, in two steps.  (1) warp w takes bins w, w + 32, ...: lane
                // (half, fl) reads its copy of cell (bin, fl) (32 lanes, 32 banks),
                // the halves' digit sums are added across the warp (a half-0 lane
                // keeps g, a half-1 lane h) and the cell's two words are held in
                // registers; once every warp has read its cells, they are written
                // over the accumulators in the staging order, feature-major:
                // word ((fl * 256 + bin) * 4 + 2 * half + {hi, lo}).  (2) the CTA
                // adds (or stores) them into staging one feature at a time, 1024
                // consecutive words per feature, so a warp covers 256 contiguous
                // bytes instead of 32 features' lines.
                long long fw[2 * (kBins / (kHistV3Threads / 32))];
#pragma unroll
                for (int i = 0; i < kBins / (kHistV3Threads / 32); i++) {
                    const int b = warp + i * (kHistV3Threads / 32);
                    const unsigned *d = acc + (b * 2 + half) * kBlk + fl;
                    const unsigned g0 = d[0], g1 = d[kDigV3], g2 = d[2 * kDigV3];
                    const unsigned h0 = d[3 * kDigV3], h1 = d[4 * kDigV3], h2 = d[5 * kDigV3];
                    // send the partner what it keeps: half 0 sends h, half 1 sends g
                    const unsigned s0 = half ? g0 : h0, s1 = half ? g1 : h1, s2 = half ? g2 : h2;
                    const unsigned r0_ = __shfl_xor_sync(0xffffffffu, s0, 16);
                    const unsigned r1_ = __shfl_xor_sync(0xffffffffu, s1, 16);
                    const unsigned r2_ = __shfl_xor_sync(0xffffffffu, s2, 16);
                    const unsigned long long lo64 = (unsigned long long)(half ? h0 : g0) + r0_;
                    const unsigned long long mid64 = (unsigned long long)(half ? h1 : g1) + r1_;
                    const long long top = (long long)(int)(half ? h2 : g2) + (long long)(int)r2_;
                    const unsigned long long a = (mid64 << kDig) + lo64;
                    fw[2 * i] = 4 * top + (long long)(a >> 32);
                    fw[2 * i + 1] = (long long)(a & 0xffffffffull);
                }
                __syncthreads();   // every cell has been read: the accumulators become the buffer
                long long *fbuf = reinterpret_cast<long long *>(acc);   // [16][256][4], 128 KB
#pragma unroll
                for (int i = 0; i < kBins / (kHistV3Threads / 32); i++) {
                    const int b = warp + i * (kHistV3Threads / 32);
                    *reinterpret_cast<longlong2 *>(fbuf + ((int64_t)fl * kBins + b) * kWords + 2 * half) =
                        make_longlong2(fw[2 * i], fw[2 * i + 1]);
                }
                __syncthreads();
                for (int f = 0; f < kBlk; f++) {
                    if (!((mask >> f) & 1u)) continue;
                    const int jj = COMPACT ? bi * kBlk + f : fpos[blk * kBlk + f];
                    long long *o = dst + (int64_t)jj * kBins * kWords;
                    const long long *src = fbuf + (int64_t)f * kBins * kWords;
                    for (int i = threadIdx.x; i < kBins * kWords; i += kHistV3Threads) {
                        const long long x = src[i];
                        if (single) o[i] = x;
                        else if (x) atomicAdd((unsigned long long *)(o + i), (unsigned long long)x);
                    }
                }
                __syncthreads();
            }
            k = pe;
        }
    }
}

// ===========================================================================
// level planning (device side: no host round trip inside a tree)
// ===========================================================================

__device__ __forceinline__ DNode fresh_node(int depth, int parent) {
    DNode d;
    d.begin = d.end = d.n = d.nl = d.gnl = 0;
    d.G = d.H = 0.0;
    d.gain = -1.0;
    d.feat = -1;
    d.bin = 0;
    d.depth = depth;
    d.parent = parent;
    d.kid0 = d.kid1 = -1;
    d.left_small = 0;
    d.expanded = 0;
    d.nan_right = 0;
    d.pad = 0;
    d.mg = -INFINITY;
    return d;
}

// Root: node 0 holds all in-bag rows; one histogram task over them.
// With several ranks (stage_count != null) node 0's count is this rank's
// until k_fill_counts puts the all-reduced one in; the rank's count goes into
// the root staging slot's count word, summed with the histogram.
__global__ void k_root_plan(const int32_t *__restrict__ n_local, const long long *__restrict__ n_global,
                            DNode *__restrict__ nodes, HistTask *__restrict__ ht,
                            int32_t *__restrict__ prefix, int *__restrict__ node_count,
                            long long *__restrict__ stage_count, const unsigned long long *__restrict__ par_word,
                            int64_t par_stride) {
    griddep_wait();
    if (threadIdx.x || blockIdx.x) return;
    long long ns = *n_local;
    if (stage_count) stage_count[par_word ? (int64_t)(*par_word & 1ull) * par_stride : 0] = ns;
    DNode d = fresh_node(0, -1);
    d.begin = 0;
    d.end = ns;
    d.n = n_global ? *n_global : ns;
    nodes[0] = d;
    HistTask t;
    t.begin = 0;
    t.end = ns;
    t.stage = 0;
    t.left_small = 1;
    t.buf = 0;
    t.pad = 0;
    ht[0] = t;
    prefix[0] = 0;
    prefix[1] = (int32_t)ns;
    *node_count = 1;
}

// Partition tasks for the parents lvl[0..W) and node ids for their children
// (children of lvl[k] are base+2k (left) and base+2k+1 (right)).  W is cut
// to the level's launch bound and to the node capacity; parents cut off stay
// unexpanded (the host expands them on demand if the replay needs them).
__global__ void k_lvl_plan(DNode *__restrict__ nodes, const int *__restrict__ lvl, int *__restrict__ lvl_count,
                           int *__restrict__ node_count, PartTask *__restrict__ pt,
                           int *__restrict__ tiles_total, int nmax, int w_max) {
    griddep_wait();
    __shared__ int s_w[32];
    __shared__ int s_W, s_base;
    if (threadIdx.x == 0) {
        int W = *lvl_count, base = *node_count;
        int cap = (nmax - base) / 2;
        if (W > w_max) W = w_max;          // the launch bounds of this level
        if (W > cap) W = cap < 0 ? 0 : cap;
        s_W = W;
        s_base = base;
    }
    __syncthreads();
    const int W = s_W, base = s_base;
    int carry = 0;
    for (int b0 = 0; b0 < W; b0 += blockDim.x) {
        int k = b0 + threadIdx.x;
        int nt = 0;
        int i = -1;
        if (k < W) {
            i = lvl[k];
            long long sz = nodes[i].end - nodes[i].begin;
            nt = (int)((sz + kPartTile - 1) / kPartTile);
            if (nt < 1) nt = 1;
        }
        int tot;
        int e = block_excl_scan(nt, s_w, tot);
        if (k < W) {
            DNode &p = nodes[i];
            PartTask t;
            t.begin = p.begin;
            t.end = p.end;
            t.feat = p.feat;
            t.thr = p.bin;
            t.tile0 = carry + e;
            t.ntile = nt;
            t.src = p.depth & 1;
            t.nan_right = p.nan_right;
            pt[k] = t;
            int c0 = base + 2 * k;
            p.kid0 = c0;
            p.kid1 = c0 + 1;
            nodes[c0] = fresh_node(p.depth + 1, i);
            nodes[c0 + 1] = fresh_node(p.depth + 1, i);
        }
        carry += tot;
    }
    if (threadIdx.x == 0) {
        *lvl_count = W;
        *node_count = base + 2 * W;
        *tiles_total = carry;
    }
}

__device__ __forceinline__ int find_task_by_tile(const PartTask *tasks, int ntask, int tile) {
    int lo = 0, hi = ntask - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (tasks[mid].tile0 <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Best-first pruning after a level's partition (one rank, full speculation;
// the rule of k_level_close, stronger here because this level's parents are
// partitioned too, so their own splits count): a parent the reference's loop
// can never split -- too many splits certain to come first, or a split that
// cannot be made (min_samples_leaf, gain <= gamma) on its path -- leaves the
// level list before its children are histogrammed or searched.  Returns the new list length; s_orig[k] is the
// kept parent k's index in the old list.  W <= kPruneList.
constexpr int kPruneList = 1024;
constexpr int kPruneTable = 2048;
__device__ int prune_parents(DNode *__restrict__ nodes, int *__restrict__ lvl, int W,
                             const long long *__restrict__ gnl_of, int ncount, double gamma, long long msl,
                             int max_leaves, double *s_mg, int *s_par, int *s_orig, int *s_w) {
    for (int k = threadIdx.x; k < W; k += blockDim.x) {
        DNode &p = nodes[lvl[k]];
        const long long gnl = gnl_of[k];
        const bool valid = p.feat >= 0 && p.gain > gamma && gnl >= msl && p.n - gnl >= msl;
        const double up = p.parent >= 0 ? nodes[p.parent].mg : INFINITY;
        p.mg = valid ? fmin(up, p.gain) : -INFINITY;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ncount; i += blockDim.x) {
        s_mg[i] = nodes[i].mg;
        s_par[i] = nodes[i].parent;
    }
    __syncthreads();
    int carry = 0;
    for (int b0 = 0; b0 < W; b0 += blockDim.x) {
        const int k = b0 + threadIdx.x;
        int keep = 0, id = -1;
        if (k < W) {
            id = lvl[k];
            const double g = nodes[id].gain;
            int cnt = 0;
            for (int i = 0; i < ncount; i++) cnt += s_mg[i] > g ? 1 : 0;
            cnt -= s_mg[id] > g ? 1 : 0;                 // not the node itself
            int depth = 0;
            for (int a = s_par[id]; a >= 0; a = s_par[a]) {
                cnt -= s_mg[a] > g ? 1 : 0;           // ancestors count once, in depth
                depth++;
            }
            // a parent whose split cannot be made, or that sits under one, is never split either
            keep = s_mg[id] > -INFINITY && depth + cnt < max_leaves - 1 ? 1 : 0;
        }
        int tot;
        const int e = block_excl_scan(keep, s_w, tot);
        if (keep) s_orig[carry + e] = k;
        carry += tot;
    }
    __syncthreads();
    for (int k = threadIdx.x; k < carry; k += blockDim.x) s_par[k] = lvl[s_orig[k]];   // the kept ids
    __syncthreads();
    for (int k = threadIdx.x; k < carry; k += blockDim.x) lvl[k] = s_par[k];
    __syncthreads();
    return carry;
}

// Level plan after the partition: each parent's smaller child (by global
// count) becomes a histogram task; the children get their row ranges.
// gl == null (several ranks): each rank histograms its locally smaller child;
// k_stage_left turns that into the left child's partial before the all-reduce
// and k_fill_counts sets the children's global counts after it.
// One CTA (the last of k_partition to finish) runs it.
__device__ void plan_hist_block(DNode *__restrict__ nodes, const int *__restrict__ lvl, int W,
                                const long long *__restrict__ nl_local, const long long *__restrict__ gl,
                                HistTask *__restrict__ ht, int32_t *__restrict__ prefix, int *s_w,
                                const int *s_orig = nullptr) {
    int carry = 0;
    for (int b0 = 0; b0 < W; b0 += blockDim.x) {
        int k = b0 + threadIdx.x;
        int ch = 0;
        if (k < W) {
            int i = lvl[k];
            DNode &p = nodes[i];
            const int ko = s_orig ? s_orig[k] : k;   // the parent's index in the partition's list
            long long nl = nl_local[ko];
            long long gnl = gl ? gl[ko] : nl, gtot = gl ? p.n : p.end - p.begin;
            bool ls = gnl <= gtot - gnl;
            HistTask t;
            t.begin = ls ? p.begin : p.begin + nl;
            t.end = ls ? p.begin + nl : p.end;
            t.stage = k;
            t.left_small = ls ? 1 : 0;
            t.buf = (p.depth + 1) & 1;
            t.pad = 0;
            ht[k] = t;
            ch = (int)(t.end - t.begin);
            p.nl = nl;
            p.gnl = gnl;
            p.left_small = t.left_small;
            DNode &a = nodes[p.kid0];
            DNode &c = nodes[p.kid1];
            a.begin = p.begin;
            a.end = p.begin + nl;
            a.n = gnl;
            c.begin = p.begin + nl;
            c.end = p.end;
            c.n = gtot - gnl;
        }
        int tot;
        int e = block_excl_scan(ch, s_w, tot);
        if (k < W) prefix[k] = carry + e;
        carry += tot;
    }
    if (threadIdx.x == 0) prefix[W] = carry;
}

// The partition of a level (the sides of E:663-674: goes_left on the split's
// feature, bin and NaN direction), in one pass.  A CTA per tile of
// kPartTile consecutive positions of a parent's row list; tiles are taken
// in order from a ticket, so every tile a CTA waits on has started.  Each
// thread holds 8 rows with their loads in flight together; the ballots of
// the tile give each row its rank among the tile's lefts, and the tile's
// left count is published for decoupled look-back: the tile's lefts before
// it in the task come from its predecessors' published sums.  Lefts are
// written to the front of the parent's range in list order, rights to its
// back in reverse order: a node's list is then ascending or descending
// (every list stays monotonic), and the order inside a node changes no
// result, every sum over it being exact.  The task's last tile stores the
// task's left count.  The last CTA to finish clears the tile words and the
// ticket for the next level and plans the children's histograms.
// A look-back wait is bounded: past kLookbackSpins polls it records the
// failure in *err (the round then fails on the host) and goes on.
constexpr unsigned long long kTileAgg = 1ull << 62, kTilePre = 2ull << 62, kTileVal = (1ull << 62) - 1;
constexpr int kLookbackSpins = 1 << 22;

// Warp 0 of a tile: the decoupled look-back over the tiles first .. tile - 1,
// 32 predecessors at a time.  Publishes this tile's aggregate `tot`, sums the
// predecessors back to the nearest one that has published its inclusive
// prefix, publishes its own and returns the exclusive prefix (the first tile
// publishes at once and returns 0).  A wait past kLookbackSpins polls sets
// *err and publishes what it summed.
__device__ __forceinline__ long long lookback_warp(volatile unsigned long long *vst, int tile, int first,
                                                   long long tot, int *err) {
    const int lane = threadIdx.x & 31;
    if (tile == first) {
        if (lane == 0) vst[tile] = kTilePre | (unsigned long long)tot;
        return 0;
    }
    if (lane == 0) vst[tile] = kTileAgg | (unsigned long long)tot;
    long long lcar = 0;
    int top = tile - 1;   // the window's nearest tile; lane l reads tile top - l
    bool bad = false;
    while (true) {
        const int j = top - lane;
        // tiles before the first (which publishes its prefix at once) add nothing
        unsigned long long v = kTilePre + 0ull;
        if (j >= first) v = vst[j];
        int spins = 0;
        while (!__all_sync(0xffffffffu, (v >> 62) != 0ull)) {
            if (++spins > kLookbackSpins) { bad = true; break; }
            if (spins > 64) __nanosleep(32);
            if ((v >> 62) == 0ull) v = vst[j];
        }
        if (bad) break;
        const unsigned pre = __ballot_sync(0xffffffffu, (v >> 62) == 2ull);
        const int k = pre ? __ffs(pre) - 1 : 31;   // the nearest tile with a prefix, else the window
        long long x = lane <= k ? (long long)(v & kTileVal) : 0ll;
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        lcar += x;
        if (pre) break;
        top -= 32;
    }
    if (bad && lane == 0) atomicExch(err, 1);
    if (lane == 0) vst[tile] = kTilePre | (unsigned long long)(lcar + tot);
    return lcar;
}

// In-bag compaction in one pass: mask -> ascending row ids, *total = their
// count.  Tiles of kCompTile rows (16 mask bytes per thread, one 16-byte
// load) are handed out in order by a ticket; a block scan ranks the in-bag
// rows inside the tile, the look-back gives the tile's offset, and the ids
// are staged in shared memory so that the stores are contiguous.  ctl holds
// [ticket, done]; the last CTA to finish zeroes the tile words and ctl.
constexpr int kCompThreads = kCompTile / 16;

__global__ void __launch_bounds__(kCompThreads)
k_compact_rows(const uint8_t *__restrict__ mask, int64_t n, int32_t *__restrict__ rows, int32_t *__restrict__ total,
               unsigned long long *__restrict__ tile_st, unsigned *__restrict__ ctl, int *__restrict__ err) {
    griddep_wait();
    __shared__ int s_out[kCompTile];
    __shared__ int s_w[32];
    __shared__ int s_tile, s_last;
    __shared__ long long s_off;
    if (threadIdx.x == 0) s_tile = (int)atomicAdd(ctl, 1u);
    __syncthreads();
    const int tile = s_tile;
    const int64_t base = (int64_t)tile * kCompTile + 16 * threadIdx.x;
    unsigned bits = 0u;
    if (base + 16 <= n) {
        const uint4 v = *reinterpret_cast<const uint4 *>(mask + base);
        const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 16; k++) bits |= (((w[k >> 2] >> (8 * (k & 3))) & 0xffu) != 0u ? 1u : 0u) << k;
    } else {
        for (int k = 0; k < 16 && base + k < n; k++) bits |= (mask[base + k] != 0 ? 1u : 0u) << k;
    }
    int tot;
    const int e = block_excl_scan(__popc(bits), s_w, tot);
    for (int k = 0, o = e; k < 16; k++)
        if ((bits >> k) & 1u) s_out[o++] = (int)(base + k);
    if (threadIdx.x < 32) {
        const long long off = lookback_warp(tile_st, tile, 0, tot, err);
        if (threadIdx.x == 0) {
            s_off = off;
            if (tile == (int)gridDim.x - 1) *total = (int32_t)(off + tot);
        }
    }
    __syncthreads();
    const long long off = s_off;
    for (int k = threadIdx.x; k < tot; k += blockDim.x) rows[off + k] = s_out[k];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(ctl + 1, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) tile_st[i] = 0ull;
    if (threadIdx.x == 0) {
        ctl[0] = 0u;
        ctl[1] = 0u;
    }
}

__global__ void __launch_bounds__(kPartThreads)
k_partition(const uint8_t *__restrict__ xb, int64_t n, int32_t *__restrict__ rows0, int32_t *__restrict__ rows1,
            const PartTask *__restrict__ tasks, const int *__restrict__ ntask_p, const int *__restrict__ tiles_total,
            unsigned long long *__restrict__ tile_st, unsigned *__restrict__ ticket, int *__restrict__ err,
            long long *__restrict__ n_left, const int32_t *__restrict__ bigidx, const uint32_t *__restrict__ topbits,
            DNode *__restrict__ nodes, const int *__restrict__ lvl, const long long *__restrict__ gl,
            HistTask *__restrict__ ht, int32_t *__restrict__ prefix, unsigned *__restrict__ done, int prune,
            const int *__restrict__ node_count, double gamma, long long msl, int max_leaves) {
    griddep_wait();
    constexpr int J = kPartTile / kPartThreads;
    constexpr int NW = kPartTile / 32;   // ballot words of a tile
    __shared__ int s_pre[NW];             // lefts before each word of the tile
    __shared__ int s_tile, s_tot;
    __shared__ long long s_lcar;
    __shared__ int s_last;
    __shared__ int s_w[32];
    if (threadIdx.x == 0) s_tile = (int)atomicAdd(ticket, 1u);
    __syncthreads();
    const int tile = s_tile;
    const int ntiles = *tiles_total;
    if (tile < ntiles) {
        const int t = find_task_by_tile(tasks, *ntask_p, tile);
        const PartTask tk = tasks[t];
        const int32_t *__restrict__ src = tk.src ? rows1 : rows0;
        int32_t *__restrict__ dst = tk.src ? rows0 : rows1;
        const long long r0 = tk.begin + (long long)(tile - tk.tile0) * kPartTile;
        const int m = (int)min((long long)kPartTile, tk.end - r0);
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        // position o = threadIdx.x + j * kPartThreads; word (o >> 5) = warp + j * (kPartThreads / 32)
        int rw[J];
#pragma unroll
        for (int j = 0; j < J; j++) {
            const int o = threadIdx.x + j * kPartThreads;
            rw[j] = o < m ? src[r0 + o] : -1;
        }
        unsigned wd[J];
#pragma unroll
        for (int j = 0; j < J; j++) {
            // threshold 255 of a 257-bin feature: the rows of bin 256 (stored as 255) go right
            const bool left = rw[j] >= 0 && goes_left(bin_of(xb, n, rw[j], tk.feat), tk.thr, tk.nan_right) &&
                              !(tk.thr >= 255 && top_bit(topbits, (n + 31) >> 5, bigidx[tk.feat], rw[j]));
            wd[j] = __ballot_sync(0xffffffffu, left);
            if (lane == 0) s_pre[warp + j * (kPartThreads / 32)] = __popc(wd[j]);
        }
        __syncthreads();
        if (warp == 0) {   // exclusive scan of the NW word counts, NW / 32 per lane
            constexpr int PER = NW / 32;
            int v[PER], sum = 0;
#pragma unroll
            for (int k = 0; k < PER; k++) { v[k] = s_pre[lane * PER + k]; sum += v[k]; }
            int incl = sum;
            for (int o = 1; o < 32; o <<= 1) {
                const int x = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += x;
            }
            int run = incl - sum;
#pragma unroll
            for (int k = 0; k < PER; k++) { s_pre[lane * PER + k] = run; run += v[k]; }
            if (lane == 31) s_tot = incl;
        }
        __syncthreads();
        if (warp == 0) {   // decoupled look-back over the task's earlier tiles
            const long long tot = s_tot;
            const long long lcar = lookback_warp(tile_st, tile, tk.tile0, tot, err);
            if (lane == 0) {
                s_lcar = lcar;
                if (tile == tk.tile0 + tk.ntile - 1) n_left[t] = lcar + tot;
            }
        }
        __syncthreads();
        const long long lcar = s_lcar;
        const long long rcar = (r0 - tk.begin) - lcar;   // rights of the task's earlier tiles
        const unsigned lt = (1u << lane) - 1u;
#pragma unroll
        for (int j = 0; j < J; j++) {
            if (rw[j] < 0) continue;
            const int o = threadIdx.x + j * kPartThreads;
            const int wi = warp + j * (kPartThreads / 32);
            const int lrank = s_pre[wi] + __popc(wd[j] & lt);   // lefts before position o in the tile
            if ((wd[j] >> lane) & 1u) dst[tk.begin + lcar + lrank] = rw[j];
            else dst[tk.end - 1 - rcar - (o - lrank)] = rw[j];
        }
    }
    // the last CTA to finish resets the tile words and plans the children's histograms
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < ntiles; i += blockDim.x) tile_st[i] = 0ull;
    if (threadIdx.x == 0) {
        *done = 0;
        *ticket = 0;
    }
    const int W = *ntask_p;
    const int ncount = prune ? *node_count : 0;
    if (prune && gl && W <= kPruneList && ncount <= kPruneTable && ncount >= max_leaves) {
        __shared__ double s_mg[kPruneTable];
        __shared__ int s_par[kPruneTable];
        __shared__ int s_orig[kPruneList];
        const int W2 = prune_parents(nodes, const_cast<int *>(lvl), W, gl, ncount, gamma, msl, max_leaves, s_mg,
                                     s_par, s_orig, s_w);
        if (threadIdx.x == 0) *const_cast<int *>(ntask_p) = W2;
        plan_hist_block(nodes, lvl, W2, n_left, gl, ht, prefix, s_w, s_orig);
        return;
    }
    plan_hist_block(nodes, lvl, W, n_left, gl, ht, prefix, s_w);
}




// ---------------------------------------------------------------------------
// several ranks: the staging exchange
//
// Every histogram level ends with the sum over ranks of the staging slots.
// With NCCL that is one all-reduce of the slots.  With the peer exchange
// each rank keeps two local staging buffers (level parity, from the level
// counter in its sync words) that all ranks map through CUDA IPC: a rank
// converts its partials in place and signals every peer (k_stage_left); each
// rank then waits for every peer's signal and pulls the level's slots from
// all ranks over NVLink, summing them into its own d_stage (k_peer_sum).  A
// level's buffer is written again two levels later, after the next level's
// signals prove that every peer has finished reading it; k_peer_sum zeroes it
// then.  Sync words of a rank (unsigned 64-bit): [0, N) signals received from
// each rank (written by the peers), then kSyncSent (signals this rank sent),
// kSyncCta (CTAs done, for the last-CTA signal), kSyncLevel (levels done),
// kSyncErr (a wait ran out), kSyncPrevW (slots of the previous level),
// kSyncWaitNs (time CTA 0 of the exchange kernels spent waiting for the
// peers), kSyncSentRed / kSyncCta2 (the two-shot exchange's second signal);
// then [N + kSyncLocal, 2N + kSyncLocal) the second signals received.
//
// With more than two ranks the sum is two-shot: k_peer_reduce sums only this
// rank's 1/N of the level's words from every rank into its IPC-visible
// result buffer and signals again; k_peer_gather waits for those signals and
// copies every rank's summed share into d_stage.  Per rank 2 (N-1)/N of the
// level crosses NVLink instead of (N-1) times it.
// ---------------------------------------------------------------------------
constexpr int kSyncSent = 0, kSyncCta = 1, kSyncLevel = 2, kSyncErr = 3, kSyncPrevW = 4, kSyncWaitNs = 5,
              kSyncSentRed = 6, kSyncCta2 = 7, kSyncLocal = 8;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Slot k holds this rank's partial histogram of the child it built (the
// locally smaller one).  Make it the LEFT child's partial -- parent - right
// when the right child was built, from this rank's own partials of earlier
// levels (lpool) -- so that every rank contributes the same child; store both
// children's partials in lpool (children that will be parents only) and this
// rank's left count in the slot's count word.  lvl == null: the root, whose
// partial is copied to lpool[0].  Integer words throughout: exact.  With the
// peer exchange (sync != null) the slots are in this level's parity buffer,
// and the last CTA to finish signals every peer.
__global__ void k_stage_left(const DNode *__restrict__ nodes, const int *__restrict__ lvl,
                             const int *__restrict__ lvl_count, HistTask *__restrict__ ht,
                             long long *__restrict__ stage, int64_t par_stride, long long *__restrict__ lpool, int nf,
                             int pool_depth, unsigned long long *__restrict__ sync,
                             unsigned long long *const *__restrict__ peer_sync, int rank, int nranks) {
    griddep_wait();
    if (sync) stage += (int64_t)(sync[nranks + kSyncLevel] & 1ull) * par_stride;
    const int k = blockIdx.y;
    const int64_t words = slot_words_for(nf);
    const int64_t data = (int64_t)nf * kBins * kWords + 4;   // cells and totals
    const int64_t tops = (int64_t)nf * kWords;              // then the top cells
    // word i of the converted range: the cells and totals, then the top cells
    auto word = [&](int64_t i) { return i < data ? i : top_cell_offset(nf, 0) + (i - data); };
    const bool active = lvl ? k < *lvl_count : k == 0;
    if (active) {
        long long *st = stage + (int64_t)k * words;
        if (!lvl) {
            for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < data + tops;
                 i += (int64_t)gridDim.x * blockDim.x)
                lpool[word(i)] = st[word(i)];
        } else {
            const int parent = lvl[k];
            const DNode &p = nodes[parent];
            const bool built_left = p.left_small != 0;
            const bool keep = nodes[p.kid0].depth < pool_depth;
            const long long *par = lpool + (int64_t)parent * words;
            long long *lk = lpool + (int64_t)p.kid0 * words, *rk = lpool + (int64_t)p.kid1 * words;
            for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < data + tops;
                 i0 += (int64_t)gridDim.x * blockDim.x) {
                const int64_t i = word(i0);
                const long long s = st[i], pv = par[i];
                const long long left = built_left ? s : pv - s;
                st[i] = left;
                if (keep) {
                    lk[i] = left;
                    rk[i] = pv - left;
                }
            }
            if (blockIdx.x == 0 && threadIdx.x == 0) {
                st[(int64_t)nf * kBins * kWords + kCountWord] = p.nl;
                ht[k].left_small = 1;   // the split search reads the slot as the left child
            }
        }
    }
    if (!sync) return;
    // the last CTA to finish tells every peer that this rank's slots are final
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long *ctr = sync + nranks + kSyncCta;
        const unsigned long long total = (unsigned long long)gridDim.x * gridDim.y;
        if (atomicAdd(ctr, 1ull) == total - 1) {
            *ctr = 0;
            __threadfence_system();
            const unsigned long long e = sync[nranks + kSyncSent] + 1;
            sync[nranks + kSyncSent] = e;
            // word `rank` of a peer's sync words has this rank as its only writer
            for (int q = 0; q < nranks; q++)
                if (q != rank) *reinterpret_cast<volatile unsigned long long *>(peer_sync[q] + rank) = e;
            __threadfence_system();
        }
    }
}

// Thread 0: wait (bounded) until flag word `first + q` of every peer q is at
// least `want`; a wait that runs out sets kSyncErr.  Returns 1 when all came.
__device__ int wait_peers(unsigned long long *sync, int first, unsigned long long want, int rank, int nranks,
                          long long timeout_ns) {
    const unsigned long long t0 = global_ns();
    int ok = sync[nranks + kSyncErr] == 0;   // after one failed wait the rank's exchange is broken
    for (int q = 0; q < nranks && ok; q++) {
        if (q == rank) continue;
        volatile unsigned long long *f = sync + first + q;
        while (*f < want) {
            if (global_ns() - t0 > (unsigned long long)timeout_ns) {
                ok = 0;
                atomicExch(sync + nranks + kSyncErr, 1ull);
                break;
            }
            __nanosleep(200);
        }
    }
    __threadfence_system();
    if (blockIdx.x == 0) sync[nranks + kSyncWaitNs] += global_ns() - t0;
    return ok;
}

// Peer exchange: wait (bounded) until every peer has signalled this level,
// then out[i] = sum over ranks r of rank r's slot word i, read from each
// rank's parity buffer (peers over NVLink), for the level's slots; zero this
// rank's other parity buffer (the previous level's, read by every peer by
// now).  A wait that runs out sets kSyncErr and the sums are not used.
__global__ void __launch_bounds__(256) k_peer_sum(const long long *const *__restrict__ peers, int64_t par_stride,
                                                  unsigned long long *__restrict__ sync, int rank, int nranks,
                                                  const int *__restrict__ lvl_count, int nf, long long *__restrict__ out,
                                                  long long *__restrict__ own, long long timeout_ns) {
    griddep_wait();
    __shared__ int s_ok;
    const unsigned long long level = sync[nranks + kSyncLevel];
    if (threadIdx.x == 0) s_ok = wait_peers(sync, 0, sync[nranks + kSyncSent], rank, nranks, timeout_ns);
    __syncthreads();
    const int64_t words = slot_words_for(nf);
    const int W = lvl_count ? *lvl_count : 1;
    const int64_t pr = (int64_t)(level & 1ull) * par_stride, po = (int64_t)((level & 1ull) ^ 1ull) * par_stride;
    const int64_t n2 = (int64_t)W * words / 2;   // longlong2 per level (slot words are even)
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, dt = (int64_t)gridDim.x * blockDim.x;
    // four elements per thread and pass, their loads from every rank in flight together
    constexpr int U = 4;
    for (int64_t base = t0; base < n2; base += (int64_t)U * dt) {
        long long x[U], y[U];
#pragma unroll
        for (int u = 0; u < U; u++) x[u] = y[u] = 0;
        if (s_ok) {
            for (int r = 0; r < nranks; r++) {
                const longlong2 *src = reinterpret_cast<const longlong2 *>(peers[r] + pr);
                longlong2 v[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t i = base + (int64_t)u * dt;
                    v[u] = i < n2 ? __ldcg(src + i) : make_longlong2(0, 0);   // L2 only: no stale L1 lines
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    x[u] += v[u].x;
                    y[u] += v[u].y;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t i = base + (int64_t)u * dt;
            if (i < n2) reinterpret_cast<longlong2 *>(out)[i] = make_longlong2(x[u], y[u]);   // zeros after a failed wait
        }
    }
    const int64_t z2 = (int64_t)sync[nranks + kSyncPrevW] * words / 2;
    for (int64_t i = t0; i < z2; i += dt) reinterpret_cast<longlong2 *>(own + po)[i] = make_longlong2(0, 0);
}

// Two-shot exchange, phase 1: after every peer's first signal, this rank's
// share [rank c, (rank+1) c) of the level's longlong2 words (c = ceil(n2/N))
// summed over all ranks into its result buffer; the last CTA to finish
// signals every peer again.
__global__ void __launch_bounds__(256) k_peer_reduce(const long long *const *__restrict__ peers, int64_t par_stride,
                                                     unsigned long long *__restrict__ sync,
                                                     unsigned long long *const *__restrict__ peer_sync, int rank,
                                                     int nranks, const int *__restrict__ lvl_count, int nf,
                                                     long long *__restrict__ red, long long timeout_ns) {
    griddep_wait();
    __shared__ int s_ok;
    const unsigned long long level = sync[nranks + kSyncLevel];
    if (threadIdx.x == 0) s_ok = wait_peers(sync, 0, sync[nranks + kSyncSent], rank, nranks, timeout_ns);
    __syncthreads();
    const int64_t words = slot_words_for(nf);
    const int W = lvl_count ? *lvl_count : 1;
    const int64_t pr = (int64_t)(level & 1ull) * par_stride;
    const int64_t n2 = (int64_t)W * words / 2;
    const int64_t cs = (n2 + nranks - 1) / nranks;
    const int64_t lo = min(n2, (int64_t)rank * cs), hi = min(n2, lo + cs);
    const int64_t dt = (int64_t)gridDim.x * blockDim.x;
    constexpr int U = 4;
    for (int64_t base = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < hi; base += (int64_t)U * dt) {
        long long x[U], y[U];
#pragma unroll
        for (int u = 0; u < U; u++) x[u] = y[u] = 0;
        if (s_ok) {
            for (int r = 0; r < nranks; r++) {
                const longlong2 *src = reinterpret_cast<const longlong2 *>(peers[r] + pr);
                longlong2 v[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t i = base + (int64_t)u * dt;
                    v[u] = i < hi ? __ldcg(src + i) : make_longlong2(0, 0);
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    x[u] += v[u].x;
                    y[u] += v[u].y;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t i = base + (int64_t)u * dt;
            if (i < hi) reinterpret_cast<longlong2 *>(red)[i] = make_longlong2(x[u], y[u]);
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long *ctr = sync + nranks + kSyncCta2;
        if (atomicAdd(ctr, 1ull) == (unsigned long long)gridDim.x - 1) {
            *ctr = 0;
            __threadfence_system();
            const unsigned long long e = sync[nranks + kSyncSentRed] + 1;
            sync[nranks + kSyncSentRed] = e;
            for (int q = 0; q < nranks; q++)
                if (q != rank)
                    *reinterpret_cast<volatile unsigned long long *>(peer_sync[q] + nranks + kSyncLocal + rank) = e;
            __threadfence_system();
        }
    }
}

// Two-shot exchange, phase 2: after every peer's second signal, every rank's
// summed share from its result buffer into d_stage; zero this rank's other
// parity buffer, as k_peer_sum does.
__global__ void __launch_bounds__(256) k_peer_gather(const long long *const *__restrict__ reds,
                                                     unsigned long long *__restrict__ sync, int rank, int nranks,
                                                     const int *__restrict__ lvl_count, int nf,
                                                     long long *__restrict__ out, long long *__restrict__ own,
                                                     int64_t par_stride, long long timeout_ns) {
    griddep_wait();
    __shared__ int s_ok;
    const unsigned long long level = sync[nranks + kSyncLevel];
    if (threadIdx.x == 0)
        s_ok = wait_peers(sync, nranks + kSyncLocal, sync[nranks + kSyncSentRed], rank, nranks, timeout_ns);
    __syncthreads();
    const int64_t words = slot_words_for(nf);
    const int W = lvl_count ? *lvl_count : 1;
    const int64_t n2 = (int64_t)W * words / 2;
    const int64_t cs = (n2 + nranks - 1) / nranks;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, dt = (int64_t)gridDim.x * blockDim.x;
    constexpr int U = 4;
    for (int64_t base = t0; base < n2; base += (int64_t)U * dt) {
        longlong2 v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t i = base + (int64_t)u * dt;
            v[u] = (i < n2 && s_ok) ? __ldcg(reinterpret_cast<const longlong2 *>(reds[(int)(i / cs)]) + i)
                                    : make_longlong2(0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t i = base + (int64_t)u * dt;
            if (i < n2) reinterpret_cast<longlong2 *>(out)[i] = v[u];   // zeros after a failed wait
        }
    }
    const int64_t po = (int64_t)((level & 1ull) ^ 1ull) * par_stride;
    const int64_t z2 = (int64_t)sync[nranks + kSyncPrevW] * words / 2;
    for (int64_t i = t0; i < z2; i += dt) reinterpret_cast<longlong2 *>(own + po)[i] = make_longlong2(0, 0);
}

// Several ranks, after the staging sum: the global counts from the slots'
// count words.  lvl == null: the root (slot 0).  With the peer exchange
// (sync != null) the level is closed: its slot count is kept for the next
// level's zeroing and the level counter advances.
__global__ void k_fill_counts(DNode *__restrict__ nodes, const int *__restrict__ lvl,
                              const int *__restrict__ lvl_count, const long long *__restrict__ stage, int nf,
                              unsigned long long *__restrict__ sync, int nranks) {
    griddep_wait();
    const int64_t words = slot_words_for(nf);
    const int64_t cw = (int64_t)nf * kBins * kWords + kCountWord;
    const int W = lvl ? *lvl_count : 1;
    if (!lvl) {
        if (threadIdx.x == 0) nodes[0].n = stage[cw];
    } else {
        for (int k = threadIdx.x; k < W; k += blockDim.x) {
            DNode &p = nodes[lvl[k]];
            const long long gnl = stage[(int64_t)k * words + cw];
            p.gnl = gnl;
            p.left_small = 1;
            nodes[p.kid0].n = gnl;
            nodes[p.kid1].n = p.n - gnl;
        }
    }
    if (sync && threadIdx.x == 0) {
        sync[nranks + kSyncPrevW] = (unsigned long long)W;
        sync[nranks + kSyncLevel] += 1;
    }
}

// Last level (every child at max_depth, where no node splits, E:775-777):
// the children need only their row counts and exact (G, H) -- no partition,
// no histogram, no split search.  Per parent task: [gL hi lo, hL hi lo, gR hi
// lo, hR hi lo, nL] int64 words, summed exactly over CTAs (and ranks).
constexpr int kLeafWords = 9;

// The last level's children from those sums (the same rounding as every
// other node: exact integer total -> float64 -> * 2^-S).  Reads through L2:
// the sums come from other CTAs' atomics.
__device__ __forceinline__ void leaf_finish_one(DNode *__restrict__ nodes, const int *__restrict__ lvl, int k,
                                                const long long *__restrict__ words,
                                                const long long *__restrict__ nl_local, double sc) {
    const long long *o = words + (int64_t)k * kLeafWords;
    DNode &p = nodes[lvl[k]];
    const long long nl = __ldcg(nl_local + k), gnl = __ldcg(o + 8);
    DNode &a = nodes[p.kid0];
    DNode &c = nodes[p.kid1];
    a.begin = p.begin;
    a.end = p.begin + nl;
    a.n = gnl;
    c.begin = p.begin + nl;
    c.end = p.end;
    c.n = p.n - gnl;
    a.G = __dmul_rn(i128_to_double(cell(__ldcg(o + 0), __ldcg(o + 1))), sc);
    a.H = __dmul_rn(i128_to_double(cell(__ldcg(o + 2), __ldcg(o + 3))), sc);
    c.G = __dmul_rn(i128_to_double(cell(__ldcg(o + 4), __ldcg(o + 5))), sc);
    c.H = __dmul_rn(i128_to_double(cell(__ldcg(o + 6), __ldcg(o + 7))), sc);
    a.feat = c.feat = -1;
    a.bin = c.bin = 0;
    a.gain = c.gain = -1.0;
    p.nl = nl;
    p.gnl = gnl;
    p.left_small = gnl <= p.n - gnl;
    p.expanded = 1;
}

// With `done` (one rank: nothing to sum over ranks in between) the last CTA
// to finish also finishes the children (leaf_finish_one) and resets *done;
// with several ranks k_leaf_finish does that after the exchange.
__global__ void __launch_bounds__(kPartThreads)
k_leaf_totals(const uint8_t *__restrict__ xb, int64_t n, const int32_t *__restrict__ rows0,
              const int32_t *__restrict__ rows1, const PartTask *__restrict__ tasks, const int *__restrict__ ntask_p,
              const int *__restrict__ tiles_total, const longlong2 *__restrict__ q,
              long long *__restrict__ words, long long *__restrict__ n_left, const int32_t *__restrict__ bigidx,
              const uint32_t *__restrict__ topbits, unsigned *__restrict__ done, DNode *__restrict__ nodes,
              const int *__restrict__ lvl, int S) {
    griddep_wait();
    __shared__ long long s[5][kPartThreads / 32];
    __shared__ int s_last;
    const int tile = blockIdx.x;
    if (tile < *tiles_total) {   // CTAs past the level's tiles still count in *done
        const int t = find_task_by_tile(tasks, *ntask_p, tile);
        const PartTask tk = tasks[t];
        const int32_t *__restrict__ rows = tk.src ? rows1 : rows0;
        const long long r0 = tk.begin + (long long)(tile - tk.tile0) * kPartTile;
        const int m = (int)min((long long)kPartTile, tk.end - r0);
        constexpr int J = kPartTile / kPartThreads;
        int rw[J];
#pragma unroll
        for (int j = 0; j < J; j++) {
            const int o = threadIdx.x + j * kPartThreads;
            rw[j] = o < m ? rows[r0 + o] : -1;
        }
        long long v[5] = {0, 0, 0, 0, 0};   // gL hL gR hR nL; |sum| < 4096 * 2^48
#pragma unroll
        for (int j = 0; j < J; j++) {
            if (rw[j] < 0) continue;
            const longlong2 qq = __ldg(q + rw[j]);
            const bool left = goes_left(bin_of(xb, n, rw[j], tk.feat), tk.thr, tk.nan_right) &&
                              !(tk.thr >= 255 && top_bit(topbits, (n + 31) >> 5, bigidx[tk.feat], rw[j]));
            v[left ? 0 : 2] += qq.x;
            v[left ? 1 : 3] += qq.y;
            v[4] += left;
        }
#pragma unroll
        for (int k = 0; k < 5; k++) {
            long long x = warp_sum(v[k]);
            if ((threadIdx.x & 31) == 0) s[k][threadIdx.x >> 5] = x;
        }
        __syncthreads();
        if (threadIdx.x < 5) {
            long long tot = 0;
            for (int w = 0; w < kPartThreads / 32; w++) tot += s[threadIdx.x][w];
            long long *o = words + (int64_t)t * kLeafWords;
            if (threadIdx.x < 4) {
                if (tot) {
                    atomicAdd((unsigned long long *)(o + 2 * threadIdx.x), (unsigned long long)(tot >> 32));
                    atomicAdd((unsigned long long *)(o + 2 * threadIdx.x + 1), (unsigned long long)(tot & 0xffffffffll));
                }
            } else if (tot) {
                atomicAdd((unsigned long long *)(o + 8), (unsigned long long)tot);
                atomicAdd((unsigned long long *)(n_left + t), (unsigned long long)tot);
            }
        }
    }
    if (!done) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int W = *ntask_p;
    const double sc = pow2(-S);
    for (int k = threadIdx.x; k < W; k += blockDim.x) leaf_finish_one(nodes, lvl, k, words, n_left, sc);
    if (threadIdx.x == 0) *done = 0;
}

__global__ void k_leaf_finish(DNode *__restrict__ nodes, const int *__restrict__ lvl,
                              const int *__restrict__ lvl_count, const long long *__restrict__ words,
                              const long long *__restrict__ nl_local, int S) {
    griddep_wait();
    const int W = *lvl_count;
    const double sc = pow2(-S);
    for (int k = threadIdx.x; k < W; k += blockDim.x) leaf_finish_one(nodes, lvl, k, words, nl_local, sc);
}

// ===========================================================================
// split search
// ===========================================================================

// k_split_bins: the split search (E:602-621, E:780-801) with one CTA of 256
// threads per (parent k, feature position jj) and one thread per bin, for both children at once
// (ROOT: node 0 alone).  Thread b reads bin b's staging cell (the smaller
// child, built by the histogram) and the parent's pool cell, forms both
// children's cells (larger = parent - smaller, E:740-745, exact), writes
// their pool slots when their own children will need them, and zeroes the
// staging cell it alone read.  A block-wide 128-bit prefix scan over the
// 256 bins gives every bin's left sums at once, so each thread evaluates
// one bin's gain (the reference's formula, every operation rounded as in
// E:602-621) and a block argmax picks the first maximum (lowest bin on a
// tie).
constexpr int kSplitThreads = kBins;

// Inclusive block scan of NV 128-bit values per thread (256 threads).
template <int NV>
__device__ __forceinline__ void block_scan_i128(i128 (&v)[NV], i128 (&tot)[NV], i128 *s_w /* [8][NV] */) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const i128 t = shfl_up_i128(v[j], o);
            if (lane >= o) v[j] += t;
        }
    }
    if (lane == 31) {
#pragma unroll
        for (int j = 0; j < NV; j++) s_w[w * NV + j] = v[j];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NV; j++) {
        i128 before = 0, all = 0;
        for (int u = 0; u < kSplitThreads / 32; u++) {
            const i128 x = s_w[u * NV + j];
            if (u < w) before += x;
            all += x;
        }
        v[j] += before;
        tot[j] = all;
    }
}

template <bool ROOT>
__global__ void __launch_bounds__(kSplitThreads, 4)   // 64 registers, no spills: 4 CTAs per SM
k_split_bins(const DNode *__restrict__ nodes, const int *__restrict__ lvl, const int *__restrict__ lvl_count,
             const HistTask *__restrict__ ht, long long *__restrict__ stage, long long *__restrict__ pool, int nf,
             const int32_t *__restrict__ fidx, const int32_t *__restrict__ counts,
             const uint8_t *__restrict__ nan_feat, int S, double lam, double mcw, long long msl, int max_depth,
             int pool_depth, FBest *__restrict__ fbest) {
    griddep_wait();
    constexpr int NS = ROOT ? 1 : 2;   // children searched
    __shared__ i128 s_w[(kSplitThreads / 32) * 2 * NS];
    __shared__ double s_bg[NS][kSplitThreads / 32];
    __shared__ int s_bb[NS][kSplitThreads / 32];
    __shared__ i128 s_c0[NS][2];   // bin 0's cell (the NaN bin when the feature has one)
    const int k = blockIdx.y, jj = blockIdx.x;
    if (!ROOT && k >= *lvl_count) return;
    if (jj >= nf) return;
    const int b = threadIdx.x, lane = b & 31, warp = b >> 5;
    const int64_t words = slot_words_for(nf);
    long long *st = stage + (int64_t)k * words;
    const long long *st_tot = st + (int64_t)nf * kBins * kWords;
    int parent = -1, ch[2] = {0, 0};
    bool small[2] = {true, false};
    if (!ROOT) {
        parent = lvl[k];
        const DNode &pn = nodes[parent];
        ch[0] = pn.kid0;
        ch[1] = pn.kid1;
        small[0] = ht[k].left_small != 0;
        small[1] = !small[0];
    }
    const long long *par = ROOT ? nullptr : pool + (int64_t)parent * words;
    // this bin's cells: the smaller child from staging, the larger = parent - smaller
    const int64_t cbase = ((int64_t)jj * kBins + b) * kWords;
    const longlong2 sa = *reinterpret_cast<const longlong2 *>(st + cbase);
    const longlong2 sd = *reinterpret_cast<const longlong2 *>(st + cbase + 2);
    longlong2 ca[NS], cd[NS];
#pragma unroll
    for (int s = 0; s < NS; s++) {
        if (small[s]) {
            ca[s] = sa;
            cd[s] = sd;
        } else {
            const longlong2 pa = *reinterpret_cast<const longlong2 *>(par + cbase);
            const longlong2 pd = *reinterpret_cast<const longlong2 *>(par + cbase + 2);
            ca[s] = make_longlong2(pa.x - sa.x, pa.y - sa.y);
            cd[s] = make_longlong2(pd.x - sd.x, pd.y - sd.y);
        }
    }
    // the staging cell is read by this thread only: zero it for the next level's adds
    *reinterpret_cast<longlong2 *>(st + cbase) = make_longlong2(0, 0);
    *reinterpret_cast<longlong2 *>(st + cbase + 2) = make_longlong2(0, 0);
    // the top cell (bin 256 of a 257-bin feature; zero otherwise), formed like the cells
    const int64_t tbase = top_cell_offset(nf, jj);
    const longlong2 ta = *reinterpret_cast<const longlong2 *>(st + tbase);
    const longlong2 td = *reinterpret_cast<const longlong2 *>(st + tbase + 2);
    longlong2 tca[NS], tcd[NS];
#pragma unroll
    for (int s = 0; s < NS; s++) {
        if (small[s]) {
            tca[s] = ta;
            tcd[s] = td;
        } else {
            const longlong2 pa = *reinterpret_cast<const longlong2 *>(par + tbase);
            const longlong2 pd = *reinterpret_cast<const longlong2 *>(par + tbase + 2);
            tca[s] = make_longlong2(pa.x - ta.x, pa.y - ta.y);
            tcd[s] = make_longlong2(pd.x - td.x, pd.y - td.y);
        }
    }
    DNode nd[NS];
    i128 TG[NS], TH[NS];
#pragma unroll
    for (int s = 0; s < NS; s++) {
        nd[s] = nodes[ch[s]];
        long long *pc = pool + (int64_t)ch[s] * words;
        if (nd[s].depth < pool_depth) {   // the cells; the totals always (level close)
            *reinterpret_cast<longlong2 *>(pc + cbase) = ca[s];
            *reinterpret_cast<longlong2 *>(pc + cbase + 2) = cd[s];
            if (b == 0) {
                *reinterpret_cast<longlong2 *>(pc + tbase) = tca[s];
                *reinterpret_cast<longlong2 *>(pc + tbase + 2) = tcd[s];
            }
        }
        long long t4[4];
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++)
            t4[q4] = small[s] ? st_tot[q4] : par[(int64_t)nf * kBins * kWords + q4] - st_tot[q4];
        TG[s] = cell(t4[0], t4[1]);
        TH[s] = cell(t4[2], t4[3]);
        if (jj == 0 && b < kTotWords) {
            const int64_t o = (int64_t)nf * kBins * kWords + b;
            pc[o] = small[s] ? st_tot[b] : par[o] - st_tot[b];
        }
    }
    // prefix over the bins: v = {g_0, h_0, g_1, h_1}
    i128 v[2 * NS], tot[2 * NS];
#pragma unroll
    for (int s = 0; s < NS; s++) {
        v[2 * s] = cell(ca[s].x, ca[s].y);
        v[2 * s + 1] = cell(cd[s].x, cd[s].y);
    }
    block_scan_i128<2 * NS>(v, tot, s_w);   // (its barrier: every thread has read the top cell)
    if (b == 0) {
        *reinterpret_cast<longlong2 *>(st + tbase) = make_longlong2(0, 0);
        *reinterpret_cast<longlong2 *>(st + tbase + 2) = make_longlong2(0, 0);
    }
    const int f = fidx[jj];
    const int nb = counts[f];
    // bin 255 of a 257-bin feature holds bins 255 and 256: the left sum at
    // threshold 255 leaves the top cell out
    if (nb > kBins && b == kBins - 1) {
#pragma unroll
        for (int s = 0; s < NS; s++) {
            v[2 * s] -= cell(tca[s].x, tca[s].y);
            v[2 * s + 1] -= cell(tcd[s].x, tcd[s].y);
        }
    }
    const double sc = pow2(-S);
    // the NaN-right candidates (nan_feat given: the learned NaN direction):
    // left = bins 1..b, right = the NaN bin and bins > b
    const bool nan_dir = nan_feat != nullptr && nan_feat[f] != 0;
    if (nan_dir) {
        if (b == 0) {
#pragma unroll
            for (int s = 0; s < NS; s++) {
                s_c0[s][0] = v[2 * s];
                s_c0[s][1] = v[2 * s + 1];
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int s = 0; s < NS; s++) {
        const i128 pg = v[2 * s], ph = v[2 * s + 1];
        const double Gd = __dmul_rn(i128_to_double(TG[s]), sc), Hd = __dmul_rn(i128_to_double(TH[s]), sc);
        const bool eval = nd[s].depth < max_depth && nd[s].n >= msl && Hd >= mcw && nb >= 2;
        // candidate c = 2 * bin + direction: ties go to the lower c, i.e. the
        // lower bin, then NaN-left (the reference's strict '>' over ascending bins)
        double bg = -1e9;
        int bc = -1;
        if (eval && b <= nb - 2) {
            const double parent_term = __ddiv_rn(__dmul_rn(Gd, Gd), __dadd_rn(Hd, lam));
            auto gain_of = [&](i128 gl, i128 hl, double &gain) {
                const double GL = __dmul_rn(i128_to_double(gl), sc);
                const double HL = __dmul_rn(i128_to_double(hl), sc);
                const double GR = __dmul_rn(i128_to_double(TG[s] - gl), sc);
                const double HR = __dmul_rn(i128_to_double(TH[s] - hl), sc);
                if (HL < mcw || HR < mcw) return false;
                gain = __dsub_rn(__dadd_rn(__ddiv_rn(__dmul_rn(GL, GL), __dadd_rn(HL, lam)),
                                           __ddiv_rn(__dmul_rn(GR, GR), __dadd_rn(HR, lam))),
                                 parent_term);
                return true;
            };
            double gn;
            if (gain_of(pg, ph, gn)) {
                bg = gn;
                bc = 2 * b;
            }
            if (nan_dir && b >= 1 && gain_of(pg - s_c0[s][0], ph - s_c0[s][1], gn) && (bc < 0 || gn > bg)) {
                bg = gn;
                bc = 2 * b + 1;
            }
        }
        // argmax: larger gain, ties -> lower candidate
        for (int o = 16; o > 0; o >>= 1) {
            const double og = __shfl_xor_sync(0xffffffffu, bg, o);
            const int oc = __shfl_xor_sync(0xffffffffu, bc, o);
            if (better(og, oc < 0 ? -1 : 0, oc, bg, bc < 0 ? -1 : 0, bc)) { bg = og; bc = oc; }
        }
        if (lane == 0) {
            s_bg[s][warp] = bg;
            s_bb[s][warp] = bc;
        }
    }
    __syncthreads();
    if (b < NS) {
        const int s = b;
        double bg = s_bg[s][0];
        int bb = s_bb[s][0];
        for (int u = 1; u < kSplitThreads / 32; u++)
            if (better(s_bg[s][u], s_bb[s][u] < 0 ? -1 : 0, s_bb[s][u], bg, bb < 0 ? -1 : 0, bb)) {
                bg = s_bg[s][u];
                bb = s_bb[s][u];
            }
        FBest o;
        o.gain = bg;
        o.bin = bb < 0 ? 0 : bb >> 1;
        o.valid = bb >= 0 ? 1 : 0;
        o.nan_right = bb >= 0 ? (bb & 1) : 0;
        o.pad = 0;
        fbest[(int64_t)(2 * k + s) * nf + jj] = o;
    }
}

// The end of a level, in one CTA (1024 threads):
//   1. per child (a warp each): the first best over feature positions, its
//      totals as float64, the parent marked expanded (E:775-801);
//   2. when `next` is given: the children with a split (and gain > gamma
//      when use_gamma) ranked by gain (ties -> lower node id), at most
//      min(M, capacity) of them, as the next level's list;
//   3. when `pt` is given: that list's plan -- two fresh children per parent
//      and the partition tasks (at most w_max parents) -- and, for a last
//      level (`leafw`), its zeroed count/total words.
// The staging totals of this level's tasks are zeroed (read for the last
// time by the split search).
//
// Best-first pruning (prune != 0; full speculation only).  The reference's
// loop (E:642-801) makes at most max_leaves - 1 splits and always splits the
// candidate of largest gain.  When it picks a node v, every candidate then
// has gain <= g(v), so every node w whose whole path from the root is made of
// splits that can be made (gain > gamma, both children >= min_samples_leaf)
// with gains > g(v) has been split before v, as have v's depth(v) ancestors.
// So if depth(v) + #{such w, not ancestors of v} >= max_leaves - 1, v is
// never split and needs no expansion: the replay of the grown table gives the
// same tree.  mg (DNode) holds each expanded node's smallest path gain; a
// node whose split cannot be made, or that was not expanded, has -inf.
// Only nodes already partitioned (this level's parents and above) count.
constexpr int kCloseThreads = 1024;
constexpr int kPruneNodes = 2048;   // node tables up to this size are pruned

template <bool ROOT>
__global__ void __launch_bounds__(kCloseThreads)
k_level_close(DNode *__restrict__ nodes, const int *__restrict__ lvl, const int *__restrict__ lvl_count,
              const long long *__restrict__ pool, long long *__restrict__ stage, int nf,
              const int32_t *__restrict__ fidx, const FBest *__restrict__ fbest, int S,
              int *__restrict__ next, int *__restrict__ next_count, int *__restrict__ node_count, int nmax, int M,
              double gamma, int use_gamma, PartTask *__restrict__ pt, int *__restrict__ tiles_total, int w_max,
              long long *__restrict__ leafw, long long *__restrict__ nleft, int prune, long long msl,
              int max_leaves) {
    griddep_wait();
    __shared__ double s_g[1024];
    __shared__ int s_id[1024];
    __shared__ double s_mg[kPruneNodes];
    __shared__ int s_par[kPruneNodes];
    __shared__ int s_cnt, s_W, s_base;
    __shared__ int s_w[32];
    const int W = ROOT ? 1 : *lvl_count;
    const int C = ROOT ? 1 : 2 * W;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t words = slot_words_for(nf);
    // 1. split reduce
    for (int cc = warp; cc < C; cc += kCloseThreads / 32) {
        int ch = 0, parent = -1;
        if (!ROOT) {
            parent = lvl[cc >> 1];
            ch = (cc & 1) ? nodes[parent].kid1 : nodes[parent].kid0;
        }
        const FBest *fb = fbest + (int64_t)cc * nf;
        double bg = -1e9;
        int bj = -1, bb = 0, br = 0;
        for (int jj = lane; jj < nf; jj += 32) {
            FBest o = fb[jj];
            if (o.valid && better(o.gain, jj, o.bin, bg, bj, bb)) { bg = o.gain; bj = jj; bb = o.bin; br = o.nan_right; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            double og = __shfl_xor_sync(0xffffffffu, bg, o);
            int oj = __shfl_xor_sync(0xffffffffu, bj, o);
            int ob = __shfl_xor_sync(0xffffffffu, bb, o);
            int orr = __shfl_xor_sync(0xffffffffu, br, o);
            if (better(og, oj, ob, bg, bj, bb)) { bg = og; bj = oj; bb = ob; br = orr; }
        }
        if (lane == 0) {
            const long long *t = pool + (int64_t)ch * words + (int64_t)nf * kBins * kWords;
            const double sc = pow2(-S);
            DNode &d = nodes[ch];
            d.G = __dmul_rn(i128_to_double(cell(t[0], t[1])), sc);
            d.H = __dmul_rn(i128_to_double(cell(t[2], t[3])), sc);
            d.feat = bj >= 0 ? fidx[bj] : -1;
            d.bin = bj >= 0 ? bb : 0;
            d.gain = bj >= 0 ? bg : -1.0;
            d.nan_right = bj >= 0 ? br : 0;
            if (!ROOT && (cc & 1) == 0) nodes[parent].expanded = 1;
        }
    }
    for (int i = threadIdx.x; i < W * kTotWords; i += kCloseThreads)
        stage[(int64_t)(i / kTotWords) * words + (int64_t)nf * kBins * kWords + i % kTotWords] = 0;
    if (!next) return;
    __syncthreads();
    // 2. next level list
    if (threadIdx.x == 0) s_cnt = 0;
    for (int cc = threadIdx.x; cc < C; cc += kCloseThreads) {
        int id = ROOT ? 0 : ((cc & 1) ? nodes[lvl[cc >> 1]].kid1 : nodes[lvl[cc >> 1]].kid0);
        const DNode &d = nodes[id];
        bool ok = d.feat >= 0 && (!use_gamma || d.gain > gamma);
        s_g[cc] = d.gain;
        s_id[cc] = ok ? id : -1;
    }
    __syncthreads();
    const int ncount = *node_count;
    if (!ROOT && prune) {
        // this level's parents, partitioned by now: their smallest path gain
        // (at every level: the deeper levels' counts read it along the path)
        for (int k = threadIdx.x; k < W; k += kCloseThreads) {
            DNode &p = nodes[lvl[k]];
            const bool valid = p.feat >= 0 && p.gain > gamma && p.gnl >= msl && p.n - p.gnl >= msl;
            const double up = p.parent >= 0 ? nodes[p.parent].mg : INFINITY;
            p.mg = valid ? fmin(up, p.gain) : -INFINITY;
        }
        __syncthreads();
    }
    // a candidate's count is at most ncount - 1: with fewer nodes nothing can be skipped
    if (!ROOT && prune && ncount <= kPruneNodes && ncount >= max_leaves) {
        for (int i = threadIdx.x; i < ncount; i += kCloseThreads) {
            s_mg[i] = nodes[i].mg;
            s_par[i] = nodes[i].parent;
        }
        __syncthreads();
        for (int cc = threadIdx.x; cc < C; cc += kCloseThreads) {
            const int id = s_id[cc];
            if (id < 0) continue;
            const double g = s_g[cc];
            int cnt = 0;
            for (int i = 0; i < ncount; i++) cnt += s_mg[i] > g ? 1 : 0;
            int depth = 0;
            for (int a = s_par[id]; a >= 0; a = s_par[a]) {
                cnt -= s_mg[a] > g ? 1 : 0;   // ancestors count once, in depth
                depth++;
            }
            if (depth + cnt >= max_leaves - 1) s_id[cc] = -1;
        }
        __syncthreads();
    }
    {
        int cap = (nmax - *node_count) / 2;
        int Mc = M < cap ? M : cap;
        if (Mc < 0) Mc = 0;
        for (int cc = threadIdx.x; cc < C; cc += kCloseThreads) {
            if (s_id[cc] < 0) continue;
            int rank = 0;
            for (int o = 0; o < C; o++) {
                if (s_id[o] < 0 || o == cc) continue;
                if (s_g[o] > s_g[cc] || (s_g[o] == s_g[cc] && s_id[o] < s_id[cc])) rank++;
            }
            if (rank < Mc) {
                next[rank] = s_id[cc];
                atomicAdd(&s_cnt, 1);
            }
        }
    }
    __syncthreads();
    if (!pt) {
        if (threadIdx.x == 0) *next_count = s_cnt;
        return;
    }
    // 3. plan the next level
    if (threadIdx.x == 0) {
        int Wn = s_cnt, base = *node_count;
        int cap = (nmax - base) / 2;
        if (Wn > w_max) Wn = w_max;
        if (Wn > cap) Wn = cap < 0 ? 0 : cap;
        s_W = Wn;
        s_base = base;
    }
    __syncthreads();
    const int Wn = s_W, base = s_base;
    int carry = 0;
    for (int b0 = 0; b0 < Wn; b0 += kCloseThreads) {
        int k = b0 + threadIdx.x;
        int ntl = 0;
        int i = -1;
        if (k < Wn) {
            i = next[k];
            long long sz = nodes[i].end - nodes[i].begin;
            ntl = (int)((sz + kPartTile - 1) / kPartTile);
            if (ntl < 1) ntl = 1;
        }
        int tot;
        int e = block_excl_scan(ntl, s_w, tot);
        if (k < Wn) {
            DNode &p = nodes[i];
            PartTask t;
            t.begin = p.begin;
            t.end = p.end;
            t.feat = p.feat;
            t.thr = p.bin;
            t.tile0 = carry + e;
            t.ntile = ntl;
            t.src = p.depth & 1;
            t.nan_right = p.nan_right;
            pt[k] = t;
            int c0 = base + 2 * k;
            p.kid0 = c0;
            p.kid1 = c0 + 1;
            nodes[c0] = fresh_node(p.depth + 1, i);
            nodes[c0 + 1] = fresh_node(p.depth + 1, i);
        }
        carry += tot;
    }
    if (leafw) {
        for (int i = threadIdx.x; i < Wn * kLeafWords; i += kCloseThreads) leafw[i] = 0;
        for (int i = threadIdx.x; i < Wn; i += kCloseThreads) nleft[i] = 0;
    }
    if (threadIdx.x == 0) {
        *next_count = Wn;
        *node_count = base + 2 * Wn;
        *tiles_total = carry;
    }
}

// ===========================================================================
// best-first replay on the device (E:642-823), post-prune, monotone clip
// ===========================================================================

// The fields of a grown node the replay reads, cached in shared memory.
struct RNode {
    double val, H, gain;    // leaf value -G/(H+lambda) (E:640, E:708-709), hessian sum, best gain
    long long n, local;     // rows over all ranks / on this rank
    int feat, bin, kid0, kid1, expanded, depth;
    int nanr;               // the split sends the NaN bin right
    int parent;             // -1 at the root
};

__device__ void load_rnodes(const DNode *__restrict__ nodes, int cnt, RNode *sn, double lam) {
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
        const DNode &d = nodes[i];
        RNode r;
        r.val = __ddiv_rn(-d.G, __dadd_rn(d.H, lam));
        r.H = d.H; r.gain = d.gain; r.n = d.n; r.local = d.end - d.begin;
        r.feat = d.feat; r.bin = d.bin; r.kid0 = d.kid0; r.kid1 = d.kid1; r.expanded = d.expanded; r.depth = d.depth;
        r.nanr = d.nan_right;
        r.parent = d.parent;
        sn[i] = r;
    }
    __syncthreads();
}

constexpr int kReplayLoaders = 256;   // threads that load the node table; warp 0 replays

// The finished tree -> the F-update layout and the host copy.  Post-prune
// (E:827-841: a split over two leaves with gain < gamma becomes a leaf,
// children first) and the monotone clip (E:2461-2499) run on lane 0; the
// prune pass is skipped when no split has gain < gamma.
__device__ void finish_tree(int nc, int *tf, int *tl, int *tr, long long *tt, double *tv, double *sg,
                            const RParams &P, const int *__restrict__ mono, TreeOut *__restrict__ out,
                            TreeDev *__restrict__ td, int status, long long root_rows, long long alg_rows) {
    const int lane = threadIdx.x & 31;
    if (P.part_err && *(volatile const int *)P.part_err) status = 3;
    bool prune = false;
    for (int k = lane; k < nc; k += 32) prune |= tf[k] != -1 && sg[k] < P.gamma;
    prune = __any_sync(0xffffffffu, prune);
    if (lane == 0) {
        if (prune) {
            for (int k = nc - 1; k >= 0; k--) {
                if (tf[k] != -1) {
                    int l = tl[k], r = tr[k];
                    if (tf[l] == -1 && tf[r] == -1 && sg[k] < P.gamma) { tf[k] = -1; tl[k] = -1; tr[k] = -1; }
                }
            }
        }
        if (P.has_mono) {
            for (int k = 0; k < nc; k++) {
                int f = tf[k];
                if (f < 0) continue;
                int c = mono[f];
                if (c == 0) continue;
                int l = tl[k], r = tr[k];
                if (l < 0 || r < 0) continue;
                double lv = tv[l], rv = tv[r];
                if ((c == 1 && lv > rv) || (c == -1 && lv < rv)) {
                    double m = __ddiv_rn(__dadd_rn(lv, rv), 2.0);
                    tv[l] = m;
                    tv[r] = m;
                }
            }
        }
        out->nc = nc;
        out->status = status;
        out->root_rows = root_rows;
        out->alg_rows = alg_rows;
        td->n = status ? 0 : nc;
    }
    __syncwarp();
    for (int k = lane; k < 256; k += 32) {
        bool in = k < nc;
        out->tf[k] = in ? tf[k] : -1;
        out->tl[k] = in ? tl[k] : -1;
        out->tr[k] = in ? tr[k] : -1;
        // a replay's tt holds the bin with the NaN direction in bit 32
        out->tt[k] = in ? (tt[k] & 0xffffffffll) : 0;
        out->nr[k] = in ? (int)(tt[k] >> 32) : 0;
        out->tv[k] = in ? tv[k] : 0.0;
        out->sg[k] = in ? sg[k] : 0.0;
        if (in) {
            td->feat[k] = tf[k];
            td->thr[k] = dev_thr(tt[k] & 0xffffffffll, (int)(tt[k] >> 32));
            td->left[k] = tl[k];
            td->right[k] = tr[k];
            td->val[k] = tv[k];
        }
    }
}

constexpr int kReplayMaxC = 160;    // candidate slots: max_leaves + 2 <= 129, 5 per lane

// A double as an unsigned key with the same order.
__device__ __forceinline__ unsigned long long order_key(double d) {
    unsigned long long u = (unsigned long long)__double_as_longlong(d);
    return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

// The ranked form of the best-first loop below, run by the whole block at
// once.  The loop pops, among its candidates, the one of largest key; so the
// smallest key along a popped node's path never rises from pop to pop, and
// two nodes u, v in different subtrees of their lowest common ancestor a are
// popped in the order of the smallest key on their paths below a (larger
// first), an ancestor before its descendants.  A split's number in the loop
// is then the count of makeable candidates (key > 0, both children >=
// min_samples_leaf) popped before it, which every candidate counts by
// itself in one pass over the others.  The candidates are the nodes of key
// > 0 whose ancestors are all makeable; the tree ids follow (a split of rank
// r numbers its children 1 + 2r and 2 + 2r).  Returns false, having written
// nothing, where the loop has to run: two candidates of equal key (the
// loop's slot order decides between them), an unexpanded candidate the loop
// would pop (its status 1), a root the loop keeps as a leaf, or a table
// larger than the sizes below.
constexpr int kRankC = kReplayLoaders;   // candidates ranked, one per thread
constexpr int kRankDepth = 15;           // deepest candidate (its turns fit a 32-bit code)
constexpr int kRankNodes = 2048;         // node tables ranked
constexpr int kRankSm = kRankDepth + 2;  // row stride of the path minima (odd)

__device__ __forceinline__ bool replay_ranked(const RNode *__restrict__ sn, int cnt, const RParams &P, int *tf, int *tl,
                                              int *tr, long long *tt, double *tv, double *sg, int &nc_out,
                                              long long &alg_out) {
    __shared__ int s_ci[kRankNodes];                  // node -> candidate index, -1 if none
    __shared__ int s_cl[kRankC], s_dm[kRankC], s_r[kRankC];
    __shared__ unsigned s_code[kRankC];               // the path's turns (1: kid1), the root's first, from bit 31
    __shared__ unsigned long long s_key[kRankC];
    __shared__ unsigned short s_sm[kRankC * kRankSm];  // [c][d]: smallest key rank on c's path at depths >= d
    __shared__ int s_nc, s_bad, s_ns;
    __shared__ unsigned long long s_alg;
    const RNode r0 = sn[0];
    if (cnt > kRankNodes || r0.n < P.msl || r0.H < P.mcw || r0.feat < 0) return false;
    const int K = P.max_leaves - 1;
    auto key_of = [&](const RNode &x) -> unsigned long long {
        return (x.feat >= 0 && x.gain > P.gamma) ? order_key(x.gain) : 0ull;
    };
    auto makeable = [&](const RNode &x) -> bool {
        return key_of(x) != 0ull && x.expanded && sn[x.kid0].n >= P.msl && sn[x.kid1].n >= P.msl;
    };
    if (threadIdx.x == 0) { s_nc = 0; s_bad = 0; s_ns = 0; s_alg = 0ull; }
    __syncthreads();
    // 1. the candidates
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
        s_ci[i] = -1;
        const RNode x = sn[i];
        const unsigned long long k = key_of(x);
        if (k == 0ull) continue;
        int a = x.parent;
        while (a >= 0 && makeable(sn[a])) a = sn[a].parent;
        if (a >= 0) continue;
        const int c = atomicAdd(&s_nc, 1);
        if (c >= kRankC || x.depth > kRankDepth) { s_bad = 1; continue; }
        s_ci[i] = c;
        s_cl[c] = i;
        s_key[c] = k;
        s_dm[c] = x.depth | (makeable(x) ? 0x100 : 0) | (x.expanded ? 0x200 : 0);
    }
    __syncthreads();
    if (s_bad) return false;
    const int nC = s_nc;
    // 2. each candidate's key rank (distinct unless two keys are equal)
    for (int t = threadIdx.x; t < nC; t += blockDim.x) {
        const unsigned long long kv = s_key[t];
        int kr = 0;
        bool tie = false;
#pragma unroll 8
        for (int u = 0; u < nC; u++) {
            const unsigned long long ku = s_key[u];
            tie |= (u != t) & (ku == kv);
            kr += ku < kv;
        }
        if (tie) s_bad = 1;
        s_sm[t * kRankSm + (s_dm[t] & 0xff)] = (unsigned short)kr;
    }
    __syncthreads();
    if (s_bad) return false;
    // 3. paths: turns and the smallest key rank below each depth (every
    // ancestor is a candidate; a thread writes only its own row, above its own depth)
    for (int t = threadIdx.x; t < nC; t += blockDim.x) {
        const int v = s_cl[t];
        unsigned short m = s_sm[t * kRankSm + (s_dm[t] & 0xff)];
        unsigned code = 0u;
        for (int w = v, a = sn[v].parent; a >= 0; w = a, a = sn[a].parent) {
            const int da = sn[a].depth;
            if (sn[a].kid1 == w) code |= 1u << (31 - da);
            const unsigned short ka = s_sm[s_ci[a] * kRankSm + da];
            m = ka < m ? ka : m;
            s_sm[t * kRankSm + da] = m;
        }
        s_code[t] = code;
    }
    __syncthreads();
    // 4. ranks: the makeable candidates popped before each candidate
    for (int t = threadIdx.x; t < nC; t += blockDim.x) {
        const unsigned cv = s_code[t];
        const int dmv = s_dm[t], dv = dmv & 0xff;
        const unsigned short *smv = s_sm + t * kRankSm;
        int before = 0;
        // branch-free, so that unrolled steps overlap their shared-memory loads
#pragma unroll 4
        for (int u = 0; u < nC; u++) {
            const int dmu = s_dm[u];
            const int du = dmu & 0xff;
            const int l = min(__clz(s_code[u] ^ cv), min(du, dv));   // depth of the lowest common ancestor
            const bool anc = l == du;                                  // u is an ancestor of v
            const int li = (anc || l == dv) ? 0 : l + 1;
            const bool first = anc || (l != dv && s_sm[u * kRankSm + li] > smv[li]);
            before += (u != t && (dmu & 0x100) && first) ? 1 : 0;
        }
        int r = INT_MAX;
        if (!(dmv & 0x200) && before < K) s_bad = 1;
        else if ((dmv & 0x100) && before < K) { r = before; atomicAdd(&s_ns, 1); }
        s_r[t] = r;
    }
    __syncthreads();
    if (s_bad) return false;
    // 5. the tree
    for (int k = threadIdx.x; k < 256; k += blockDim.x) { tf[k] = -1; tl[k] = -1; tr[k] = -1; tt[k] = 0; tv[k] = 0.0; sg[k] = 0.0; }
    __syncthreads();
    auto split_rank = [&](int node) -> int { const int c = s_ci[node]; return c < 0 ? INT_MAX : s_r[c]; };
    const int ns = s_ns;
    for (int t = threadIdx.x; t < nC; t += blockDim.x) {
        const int r = s_r[t];
        if (r == INT_MAX) continue;
        const int v = s_cl[t];
        const RNode &x = sn[v];
        const int p = x.parent;
        const int cur = p < 0 ? 0 : (sn[p].kid0 == v ? 1 : 2) + 2 * split_rank(p);
        tf[cur] = x.feat; tt[cur] = x.bin | ((long long)x.nanr << 32); tl[cur] = 1 + 2 * r; tr[cur] = 2 + 2 * r;
        tv[cur] = x.val; sg[cur] = x.gain;
        if (split_rank(x.kid0) == INT_MAX) tv[1 + 2 * r] = sn[x.kid0].val;
        if (split_rank(x.kid1) == INT_MAX) tv[2 + 2 * r] = sn[x.kid1].val;
        if (x.depth + 1 < P.max_depth) {   // the last level builds no histogram
            const int ks = sn[x.kid0].n <= sn[x.kid1].n ? x.kid0 : x.kid1;
            atomicAdd(&s_alg, (unsigned long long)sn[ks].local);
        }
    }
    if (ns == 0 && threadIdx.x == 0) tv[0] = r0.val;
    __syncthreads();
    nc_out = 1 + 2 * ns;
    alg_out = r0.local + (long long)s_alg;
    return true;
}

// One warp replays the reference's best-first loop over the grown node
// table: the candidate slots, the strict '>' scan where the lowest slot wins
// among equal gains, min_samples_leaf on the partition, the node numbering
// and the reuse of the two lowest free slots (E:546-823).  Slot s belongs to
// lane s % 32, which keeps its key (the gain's order key when the slot is a
// candidate with gain > gamma, else 0) in a register; the argmax is three
// warp reductions.  status 1: the loop reached a node that was not expanded
// (the caller then replays on the host).  The block first tries the ranked
// form (replay_ranked), which gives the same tree; the loop runs where it
// hands over.
__global__ void __launch_bounds__(kReplayLoaders, 1)
k_replay_leaf(const DNode *__restrict__ nodes, const int *__restrict__ node_count, RParams P,
              const int *__restrict__ mono, TreeOut *__restrict__ out, TreeDev *__restrict__ td) {
    griddep_wait();
    extern __shared__ RNode sn[];
    __shared__ int c_node[kReplayMaxC], c_nid[kReplayMaxC];
    __shared__ int tf[256], tl[256], tr[256];
    __shared__ long long tt[256];
    __shared__ double tv[256], sg[256];
    const int cnt = *node_count;
    load_rnodes(nodes, cnt, sn, P.lam);
    {
        int nc_r;
        long long alg_r;
        if (replay_ranked(sn, cnt, P, tf, tl, tr, tt, tv, sg, nc_r, alg_r)) {
            if (threadIdx.x < 32) finish_tree(nc_r, tf, tl, tr, tt, tv, sg, P, mono, out, td, 0, sn[0].local, alg_r);
            return;
        }
    }
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const unsigned full = 0xffffffffu;
    const int MAXC = P.max_leaves + 2;
    for (int k = lane; k < 256; k += 32) { tf[k] = -1; tl[k] = -1; tr[k] = -1; tt[k] = 0; tv[k] = 0.0; sg[k] = 0.0; }
    __syncwarp();
    const RNode r0 = sn[0];
    long long alg = r0.local;
    if (r0.n < P.msl || r0.H < P.mcw || r0.feat < 0) {          // E:575-579, E:634-638
        if (lane == 0) tv[0] = r0.val;
        __syncwarp();
        finish_tree(1, tf, tl, tr, tt, tv, sg, P, mono, out, td, 0, r0.local, alg);
        return;
    }
    auto cand_key = [&](const RNode &x) -> unsigned long long {
        return (x.feat >= 0 && x.gain > P.gamma) ? order_key(x.gain) : 0ull;
    };
    unsigned long long key[5];
    unsigned act = 0;                                            // bit r: slot lane + 32 r is active
#pragma unroll
    for (int r = 0; r < 5; r++) key[r] = 0ull;
    if (lane == 0) {
        c_node[0] = 0;
        c_nid[0] = 0;
        key[0] = cand_key(r0);
        act = 1u;
    }
    __syncwarp();
    int nc = 1, n_splits = 0, status = 0;
    while (n_splits < P.max_leaves - 1) {
        unsigned long long bk = 0ull;
        unsigned bs = 0xffffffffu;
#pragma unroll
        for (int r = 0; r < 5; r++)
            if (key[r] > bk) { bk = key[r]; bs = (unsigned)(lane + 32 * r); }
        const unsigned hi = __reduce_max_sync(full, (unsigned)(bk >> 32));
        const unsigned lo = __reduce_max_sync(full, (unsigned)(bk >> 32) == hi ? (unsigned)bk : 0u);
        if (hi == 0u && lo == 0u) break;
        const int ci = (int)__reduce_min_sync(full, ((unsigned)(bk >> 32) == hi && (unsigned)bk == lo) ? bs : full);
        const int cur = c_node[ci];
        const RNode pn = sn[c_nid[ci]];
        if (!pn.expanded) { status = 1; break; }
        const long long gnl = sn[pn.kid0].n, gnr = sn[pn.kid1].n;
        const int own = ci & 31, orr = ci >> 5;
        if (gnl < P.msl || gnr < P.msl) {                        // E:678-683
            if (lane == 0) { tf[cur] = -1; tv[cur] = pn.val; }
#pragma unroll
            for (int r = 0; r < 5; r++)
                if (lane == own && r == orr) { key[r] = 0ull; act &= ~(1u << r); }
            __syncwarp();
            continue;
        }
        // the two lowest free slots other than ci (E:712-720)
        int ss = -1, sl = -1;
#pragma unroll
        for (int r = 0; r < 5; r++) {
            const int s = lane + 32 * r;
            unsigned m = __ballot_sync(full, s < MAXC && s != ci && !((act >> r) & 1u));
            while (m && sl < 0) {
                const int b = __ffs(m) - 1;
                m &= m - 1;
                if (ss < 0) ss = 32 * r + b; else sl = 32 * r + b;
            }
        }
        if (ss < 0 || sl < 0) { status = 2; break; }            // cannot happen: >= 3 slots are free
        const int lid = nc, rid = nc + 1;
        nc += 2;
        n_splits++;
        const bool left_small = gnl <= gnr;
        const int kid_s = left_small ? pn.kid0 : pn.kid1, kid_l = left_small ? pn.kid1 : pn.kid0;
        if (pn.depth + 1 < P.max_depth) alg += sn[kid_s].local;   // the last level builds no histogram
        if (lane == 0) {
            tf[cur] = pn.feat; tt[cur] = pn.bin | ((long long)pn.nanr << 32); tl[cur] = lid; tr[cur] = rid; tv[cur] = pn.val; sg[cur] = pn.gain;
            c_node[ss] = left_small ? lid : rid;
            c_nid[ss] = kid_s;
            c_node[sl] = left_small ? rid : lid;
            c_nid[sl] = kid_l;
        }
        const unsigned long long ks = cand_key(sn[kid_s]), kl = cand_key(sn[kid_l]);
#pragma unroll
        for (int r = 0; r < 5; r++) {
            const int s = lane + 32 * r;
            if (s == ci) { key[r] = 0ull; act &= ~(1u << r); }
            if (s == ss) { key[r] = ks; act |= 1u << r; }
            if (s == sl) { key[r] = kl; act |= 1u << r; }
        }
        __syncwarp();
    }
    if (!status) {
#pragma unroll
        for (int r = 0; r < 5; r++) {
            if ((act >> r) & 1u) {
                const int s = lane + 32 * r;
                tf[c_node[s]] = -1;
                tv[c_node[s]] = sn[c_nid[s]].val;
            }
        }
    }
    __syncwarp();
    finish_tree(nc, tf, tl, tr, tt, tv, sg, P, mono, out, td, status, r0.local, alg);
}

// Depth-wise growth's node numbering (E:233-508): a DFS stack where the
// larger child is pushed first, so the smaller one is numbered first.
__global__ void __launch_bounds__(kReplayLoaders)
k_replay_depth(const DNode *__restrict__ nodes, const int *__restrict__ node_count, RParams P,
               const int *__restrict__ mono, TreeOut *__restrict__ out, TreeDev *__restrict__ td) {
    griddep_wait();
    extern __shared__ RNode sn[];
    __shared__ int tf[256], tl[256], tr[256];
    __shared__ long long tt[256];
    __shared__ double tv[256], sg[256];
    __shared__ int s_nc, s_status;
    __shared__ long long s_alg;
    load_rnodes(nodes, *node_count, sn, P.lam);
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    for (int k = lane; k < 256; k += 32) { tf[k] = -1; tl[k] = -1; tr[k] = -1; tt[k] = 0; tv[k] = 0.0; sg[k] = 0.0; }
    __syncwarp();
    if (lane == 0) {
        int st_nid[64], st_tid[64], sp = 0, nc = 0, status = 0;
        long long alg = sn[0].local;
        st_nid[sp] = 0; st_tid[sp] = nc++; sp++;
        while (sp > 0) {
            sp--;
            const RNode x = sn[st_nid[sp]];
            const int tid = st_tid[sp];
            const double val = x.val;
            if (x.feat >= 0 && !x.expanded) status = 1;
            bool split = x.feat >= 0 && x.expanded && sn[x.kid0].n >= P.msl && sn[x.kid1].n >= P.msl &&
                         nc + 2 <= 256 && sp + 2 <= 64;
            if (!split) { tf[tid] = -1; tv[tid] = val; continue; }
            const int lid = nc++, rid = nc++;
            const long long gl = sn[x.kid0].n, gr = sn[x.kid1].n;
            if (x.depth + 1 < P.max_depth) alg += gl <= gr ? sn[x.kid0].local : sn[x.kid1].local;
            tf[tid] = x.feat; tt[tid] = x.bin | ((long long)x.nanr << 32); tl[tid] = lid; tr[tid] = rid; tv[tid] = val; sg[tid] = x.gain;
            if (gl <= gr) {
                st_nid[sp] = x.kid1; st_tid[sp] = rid; sp++;
                st_nid[sp] = x.kid0; st_tid[sp] = lid; sp++;
            } else {
                st_nid[sp] = x.kid0; st_tid[sp] = lid; sp++;
                st_nid[sp] = x.kid1; st_tid[sp] = rid; sp++;
            }
        }
        s_nc = nc;
        s_status = status;
        s_alg = alg;
    }
    __syncwarp();
    finish_tree(s_nc, tf, tl, tr, tt, tv, sg, P, mono, out, td, s_status, sn[0].local, s_alg);
}

// ===========================================================================
// predict (ensemble traversal, E:863-884)
// ===========================================================================

// The ensemble is walked in chunks of whole consecutive trees that fit the
// shared-memory node buffer (kPredChunkNodes nodes, at most kPredChunkTrees
// trees).  k_pred_chunks cuts the trees into chunks greedily with one warp
// that tests 32 offsets per step, and writes each chunk as {first tree, end
// tree, first node, node count}; a tree larger than the buffer is a chunk of
// its own and is walked from global memory.
constexpr int kPredThreads = 768;   // 24 warps: one CTA of 1536 rows per SM at p = 100
constexpr int kPredChunkNodes = 2048;
constexpr int kPredChunkTrees = 512;

__global__ void k_pred_chunks(const int32_t *__restrict__ off, int ntree, int4 *__restrict__ chunks,
                              int32_t *__restrict__ nchunk) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    int t0 = 0, nc = 0;
    while (t0 < ntree) {
        const int base = __ldg(off + t0);
        int t1 = -1;
        for (int j = t0 + 1; t1 < 0; j += 32) {
            const int t = j + lane;
            // the first t that does not fit: chunk [t0, t) is then maximal
            bool stop = t > ntree || t - t0 > kPredChunkTrees || __ldg(off + t) - base > kPredChunkNodes;
            unsigned b = __ballot_sync(0xffffffffu, stop);
            if (b) t1 = j + __ffs(b) - 1;
        }
        t1 = max(t1 - 1, t0 + 1);
        if (lane == 0) chunks[nc] = make_int4(t0, t1, base, __ldg(off + t1) - base);
        nc++;
        t0 = t1;
    }
    if (lane == 0) *nchunk = nc;
}

__device__ __forceinline__ void cp_async4(void *sdst, const void *gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(sdst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async8(void *sdst, const void *gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(sdst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// One tree for a thread's RPT rows, PACKED format: exactly `dep` steps (a
// leaf points at itself with threshold 255, so no bin moves it).  `tn` and
// the rows are shared or global memory as the caller's pointers are; each
// call site is inlined with a known address space.  The word (pack_model):
//   bits 24-31 threshold, 23 NaN right, 21-22 feature & 3, 12-20 feature >> 2,
//   0-11 left child (the right child is left + 1);
// so the feature's byte in the swizzled row tile is at
// ((w >> 5) & 0xff80) | ((w >> 21) & 3), and the row goes right when
// (bin << 24) > w (the bits below the threshold never reach a whole step
// of it).  The features were checked below p and the children inside the
// tree when the model was packed (p is the model's feature count, checked
// again at launch), so no index is clamped here: every word comes from
// pack_model.  NR: the model has NaN-right splits (threshold stored as t - 1;
// the walk compares bin - 1 mod 256, so bin 0 goes right).
template <int RPT, bool SROWS, bool NR>
__device__ __forceinline__ void step_packed(const uint32_t *__restrict__ tn, const uint8_t *const *rowp,
                                            int *node) {
#pragma unroll
    for (int j = 0; j < RPT; j++) {
        const uint32_t w = tn[node[j]];
        uint32_t b;
        if (SROWS) {
            b = rowp[j][((w >> 5) & 0xff80u) | ((w >> 21) & 3u)];
        } else {
            const uint32_t f = ((w >> 10) & 0x7fcu) | ((w >> 21) & 3u);
            b = __ldg(rowp[j] + f);
        }
        if (NR) b = (b - ((w >> 23) & 1u)) & 0xffu;
        node[j] = (int)(w & 0xfffu) + ((b << 24) > w ? 1 : 0);
    }
}

template <int RPT, bool SROWS, bool NR>
__device__ __forceinline__ void walk_packed(const uint32_t *__restrict__ tn, int dep, const uint8_t *const *rowp,
                                            int *node) {
    if (dep == 8) {   // the common depth, unrolled
#pragma unroll
        for (int s = 0; s < 8; s++) step_packed<RPT, SROWS, NR>(tn, rowp, node);
        return;
    }
    for (int s = 0; s < dep; s++) step_packed<RPT, SROWS, NR>(tn, rowp, node);
}

// The same in the 8-byte PNode format (the reference's numbering): walk
// until every row is at a leaf, at most szm1 steps.
template <int RPT, bool SROWS>
__device__ __forceinline__ void walk_pnode(const PNode *__restrict__ tn, int szm1, int pm1,
                                           const uint8_t *const *rowp, int *node, const int64_t *rid,
                                           const int32_t *__restrict__ bigidx, const uint32_t *__restrict__ topbits,
                                           int64_t top_words) {
    PNode nd[RPT];
#pragma unroll
    for (int j = 0; j < RPT; j++) nd[j] = tn[0];
    for (int s = 0; s < szm1; s++) {
        bool more = false;
#pragma unroll
        for (int j = 0; j < RPT; j++) {
            if (nd[j].feat >= 0) {
                const int f = min((int)nd[j].feat, pm1);
                const int b = SROWS ? rowp[j][((f >> 2) << 7) | (f & 3)] : __ldg(rowp[j] + f);
                // threshold 255 on a 257-bin feature: a row of bin 256 (stored as 255) goes right
                // (unless the model's threshold is above 255: nanr bit 1)
                const bool l = goes_left(b, nd[j].thr, nd[j].nanr & 1) &&
                               !(!(nd[j].nanr & 2) && nd[j].thr == 255 && bigidx &&
                                 top_bit(topbits, top_words, bigidx[f], rid[j]));
                node[j] = min((int)(l ? nd[j].left : nd[j].right), szm1);
                nd[j] = tn[node[j]];
                more = true;
            }
        }
        if (!more) break;
    }
}

// F[i] = base + sum_t lr * value_t(leaf_t(i)), summed in tree order
// (predict_all_trees_jit, E:863-884), and proba = sigmoid(clip(F, +-500))
// (E:3318-3336).
//
// A CTA takes rpc <= RPT x kPredThreads consecutive rows.  With SROWS their bins are
// staged in shared memory once, swizzled so that the 32 lanes of a warp (32
// consecutive rows) read 32 different banks whatever features they test:
// byte f of tile row r sits at byte 4 * ((r / 32) * P4 * 32 + r % 32) +
// 128 * (f / 4) + f % 4 (P4 = ceil(p / 4)); without SROWS (rows too wide for
// shared memory) the bins are read from the row in global memory.  The
// chunks of whole trees (nodes, values, offsets, depths) stream through two
// shared-memory buffers: while the CTA walks chunk c, cp.async copies chunk
// c + 1 into the other buffer.
//
// Node formats.  PACKED: one 32-bit word per node of a tree renumbered
// breadth-first (pack_model), children adjacent: threshold, NaN direction,
// feature and left child (walk_packed), right = left + 1 (a NaN-right split
// holds threshold - 1 and compares bin - 1 mod 256, so the NaN bin goes
// right), and a leaf pointing at itself with threshold 255; every row takes
// exactly the tree's depth steps with no branch.  Level d of a complete tree is 2^d consecutive words,
// conflict-free up to level 5.  Otherwise PNode (8 bytes, the reference's
// own numbering), walked until a leaf.
//
// The walk is bounded.  PNode: whatever the node table holds, a feature is
// clamped below p, a child below the tree's size, and a walk stops after
// size - 1 steps (a valid tree's children come after their parent, so a
// real walk never needs more).  PACKED: the words are built on the host
// from a checked model (features below its feature count, which the rows
// must match, children inside the tree, leaves pointing at themselves),
// and every row takes at most min(depth, size - 1) steps.
template <bool PACKED>
struct PredBuf {
    static constexpr int kNodeBytes = PACKED ? 4 : 8;
    static constexpr size_t kBytes =
        (sizeof(double) + kNodeBytes) * kPredChunkNodes + 2 * sizeof(int32_t) * (kPredChunkTrees + 4);
};

template <int RPT, bool PACKED, bool SROWS, bool NR>
__global__ void __launch_bounds__(kPredThreads)
k_predict(const uint8_t *__restrict__ xr, int64_t n, int p, const void *__restrict__ nodes_v,
          const double *__restrict__ vals, const int32_t *__restrict__ off, const int32_t *__restrict__ depth_g,
          int ntree, const int4 *__restrict__ chunks, const int32_t *__restrict__ nchunk_p, int rpc, double lr,
          double base, double *__restrict__ F, double *__restrict__ proba, const int32_t *__restrict__ bigidx,
          const uint32_t *__restrict__ topbits) {
    extern __shared__ __align__(16) unsigned char psm[];
    constexpr int kNodeBytes = PredBuf<PACKED>::kNodeBytes;
    constexpr size_t kBuf = PredBuf<PACKED>::kBytes;
    uint8_t *s_rows = psm + 2 * kBuf;
    const int64_t r0 = (int64_t)blockIdx.x * rpc;
    if (r0 >= n) return;
    const int nr = (int)min(n - r0, (int64_t)min(rpc, kPredThreads * RPT));
    const int P4 = (p + 3) >> 2;
    const int nch = min(*nchunk_p, ntree);

    // chunk c's validated bounds; staged when it fits a buffer
    auto chunk = [&](int c, int &t0, int &t1, int &o0, int &cn) {
        const int4 d = __ldg(chunks + c);
        t0 = min(max(d.x, 0), ntree);
        t1 = min(max(d.y, t0), ntree);
        o0 = __ldg(off + t0);
        cn = __ldg(off + t1) - o0;
        return t1 > t0 && cn <= kPredChunkNodes && t1 - t0 <= kPredChunkTrees;
    };
    auto prefetch = [&](int c) {
        int t0, t1, o0, cn;
        if (!chunk(c, t0, t1, o0, cn)) return;
        unsigned char *b = psm + (c & 1) * kBuf;
        double *s_val = reinterpret_cast<double *>(b);
        unsigned char *s_nd = b + sizeof(double) * kPredChunkNodes;
        int32_t *s_off = reinterpret_cast<int32_t *>(s_nd + kNodeBytes * kPredChunkNodes);
        int32_t *s_dep = s_off + kPredChunkTrees + 4;
        for (int i = threadIdx.x; i < cn; i += kPredThreads) {
            if (PACKED)
                cp_async4(s_nd + 4 * i, reinterpret_cast<const uint32_t *>(nodes_v) + o0 + i);
            else
                cp_async8(s_nd + 8 * i, reinterpret_cast<const PNode *>(nodes_v) + o0 + i);
            cp_async8(s_val + i, vals + o0 + i);
        }
        for (int i = threadIdx.x; i <= t1 - t0; i += kPredThreads) cp_async4(s_off + i, off + t0 + i);
        if (PACKED)
            for (int i = threadIdx.x; i < t1 - t0; i += kPredThreads) cp_async4(s_dep + i, depth_g + t0 + i);
    };

    if (nch > 0) prefetch(0);
    cp_async_commit();
    if (SROWS) {   // the row tile, swizzled; whole 4-byte words when p % 4 == 0
        const uint8_t *src = xr + r0 * p;
        if ((p & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 3) == 0) {
            const uint32_t *s4 = reinterpret_cast<const uint32_t *>(src);
            uint32_t *d4 = reinterpret_cast<uint32_t *>(s_rows);
            const int words = nr * P4;
            for (int w = threadIdx.x; w < words; w += kPredThreads) {
                const int r = w / P4, fw = w - r * P4;
                d4[((r >> 5) * P4 + fw) * 32 + (r & 31)] = __ldg(s4 + w);
            }
        } else {
            const int bytes = nr * p;
            for (int b = threadIdx.x; b < bytes; b += kPredThreads) {
                const int r = b / p, f = b - r * p;
                s_rows[(((r >> 5) * P4 + (f >> 2)) * 32 + (r & 31)) * 4 + (f & 3)] = __ldg(src + b);
            }
        }
    }
    double acc[RPT];
    const uint8_t *rowp[RPT];   // the tile's byte base of the row (SROWS), else the row in global memory
    int64_t rid[RPT];           // the row's index (its top bits)
    bool live[RPT];
    const int64_t top_words = (n + 31) >> 5;
#pragma unroll
    for (int j = 0; j < RPT; j++) {
        const int r = threadIdx.x + j * kPredThreads;
        acc[j] = 0.0;
        live[j] = r < nr;
        const int rr = live[j] ? r : 0;   // a thread past the tile walks row 0 and writes nothing
        rowp[j] = SROWS ? s_rows + 4 * ((rr >> 5) * P4 * 32 + (rr & 31)) : xr + (r0 + rr) * p;
        rid[j] = r0 + rr;
    }
    const int pm1 = p - 1;
    for (int c = 0; c < nch; c++) {
        cp_async_wait_all();
        __syncthreads();   // chunk c is in its buffer; nobody still reads chunk c - 1's
        if (c + 1 < nch) prefetch(c + 1);
        cp_async_commit();
        int t0, t1, o0, cn;
        const bool staged = chunk(c, t0, t1, o0, cn);
        if (t1 <= t0) continue;
        const unsigned char *b = psm + (c & 1) * kBuf;
        const double *s_val = reinterpret_cast<const double *>(b);
        const unsigned char *s_nd = b + sizeof(double) * kPredChunkNodes;
        const int32_t *s_off = reinterpret_cast<const int32_t *>(s_nd + kNodeBytes * kPredChunkNodes);
        const int32_t *s_dep = s_off + kPredChunkTrees + 4;
        for (int t = t0; t < t1; t++) {
            int node[RPT];
#pragma unroll
            for (int j = 0; j < RPT; j++) node[j] = 0;
            double v[RPT];
            if (staged) {
                const int ob = s_off[t - t0] - o0, sz = s_off[t - t0 + 1] - o0 - ob;
                if (sz <= 0) continue;
                if (PACKED)
                    walk_packed<RPT, SROWS, NR>(reinterpret_cast<const uint32_t *>(s_nd) + ob,
                                                min(s_dep[t - t0], sz - 1), rowp, node);
                else
                    walk_pnode<RPT, SROWS>(reinterpret_cast<const PNode *>(s_nd) + ob, sz - 1, pm1, rowp, node, rid,
                                           bigidx, topbits, top_words);
#pragma unroll
                for (int j = 0; j < RPT; j++) v[j] = s_val[ob + node[j]];
            } else {
                const int ob = __ldg(off + t), sz = __ldg(off + t + 1) - ob;
                if (sz <= 0) continue;
                if (PACKED)
                    walk_packed<RPT, SROWS, NR>(reinterpret_cast<const uint32_t *>(nodes_v) + ob,
                                                min(__ldg(depth_g + t), sz - 1), rowp, node);
                else
                    walk_pnode<RPT, SROWS>(reinterpret_cast<const PNode *>(nodes_v) + ob, sz - 1, pm1, rowp, node, rid,
                                           bigidx, topbits, top_words);
#pragma unroll
                for (int j = 0; j < RPT; j++) v[j] = __ldg(vals + ob + node[j]);
            }
#pragma unroll
            for (int j = 0; j < RPT; j++) acc[j] = __dadd_rn(acc[j], __dmul_rn(lr, v[j]));
        }
    }
    cp_async_wait_all();
#pragma unroll
    for (int j = 0; j < RPT; j++) {
        if (!live[j]) continue;
        const int64_t i = r0 + threadIdx.x + j * kPredThreads;
        const double f = __dadd_rn(acc[j], base);
        if (F) F[i] = f;
        if (proba) {
            const double cl = fmin(fmax(f, -500.0), 500.0);
            proba[i] = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-cl)));
        }
    }
}

// Shared memory of a k_predict launch with rows_per_cta rows of p bytes:
// two chunk buffers, then the swizzled tile (whole 32-row groups of
// ceil(p / 4) words).
inline size_t predict_smem(int rows_per_cta, int p, bool packed) {
    return 2 * (packed ? PredBuf<true>::kBytes : PredBuf<false>::kBytes) +
           (size_t)((rows_per_cta + 31) / 32) * 32 * 4 * ((p + 3) / 4);
}

}  // namespace gbm
