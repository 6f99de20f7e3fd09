// gbm_b200.cu -- B200 engine for the reference's binary-logloss boosting round.
//
// One boosting round of HybridHistGBMNumbaV1_0_1._fit_binary
// (src/bsscl_gbm/estimator_v1_0_1.py, "E" below, E:2849-2905) runs here:
//
//   k_update      F += lr * leaf(tree, row) for every row (E:2896-2897),
//                 the train logloss (E:2905, E:2320-2325) and the next
//                 round's fixed-point gradient/hessian (E:2861, E:2873-2874)
//                 fused in one pass over the rows.
//   k_hist        per-node (g, h) histograms over column-blocked uint8 bins
//                 (E:582-596, E:723-737): 16-byte row loads, shared-memory
//                 int64 accumulators per CTA, exact flush into global
//                 (hi, lo) int64 words.
//   k_finish      sibling subtraction: the larger child = parent - smaller
//                 (E:740-745), exact.
//   k_split       best (feature, bin) per node with the reference's gain and
//                 scan order (E:602-621, E:780-801): warp prefix scans of the
//                 exact 128-bit sums.
//   k_part_*      stable partition of a node's row list on bin <= threshold
//                 (E:663-674).
//   k_predict     the packed-ensemble traversal of predict_proba (E:863-884).
//
// Exactness.  Every g and h is rounded once to the grid 2^-S and all sums
// are integer sums, so every histogram, total and gain is independent of
// row order, CTA schedule and GPU count.  A CTA adds at most kChunk rows
// into one int64 shared-memory cell; S is chosen so that such a partial sum
// cannot overflow.  Each partial P is flushed as two independent int64
// words (P >> 32, P & 0xffffffff) whose sums never overflow and recombine
// exactly to the 128-bit total.  NCCL sums those words over ranks.
//
// The best-first order of the reference (E:642-813) is replayed on the host
// from per-node results; nodes are expanded on the device in batched waves.

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/gbm_b200.h"
#include "comm.h"

namespace {

constexpr int kBins = 256;          // uint8 bin ids
constexpr int kBlk = 16;            // features per column block (one 16-byte load)
constexpr int kWords = 4;           // g_hi, g_lo, h_hi, h_lo per histogram cell
constexpr int kChunk = 16384;       // max rows one CTA adds into one cell (R_max)
constexpr int kHistThreads = 512;
constexpr int kPartTile = 4096;     // rows per partition CTA
constexpr int kPartThreads = 256;
constexpr int kSplitThreads = 256;
constexpr int kMaxWave = 256;       // nodes expanded per wave
constexpr int kUpdThreads = 256;

typedef __int128 i128;

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ double pow2(int e) {
    return __longlong_as_double((long long)(1023 + e) << 52);
}

// Correctly rounded (nearest-even) 128-bit integer -> double.
__device__ __forceinline__ double i128_to_double(i128 v) {
    bool neg = v < 0;
    unsigned __int128 m = neg ? (unsigned __int128)(-v) : (unsigned __int128)v;
    unsigned long long hi = (unsigned long long)(m >> 64);
    unsigned long long lo = (unsigned long long)m;
    double r;
    if (hi == 0) {
        r = __ull2double_rn(lo);
    } else {
        int sh = 64 - __clzll((long long)hi);                  // 1..64
        unsigned long long top = (unsigned long long)(m >> sh); // bit 63 set
        unsigned long long rest = (sh == 64) ? lo : (lo & ((1ull << sh) - 1ull));
        if (rest) top |= 1ull;                                  // sticky
        r = __dmul_rn(__ull2double_rn(top), pow2(sh));
    }
    return neg ? -r : r;
}

__device__ __forceinline__ i128 cell(long long hi, long long lo) {
    return ((i128)hi << 32) + (i128)lo;
}

// p = 1/(1+exp(-clip(F,-500,500))), g = w(p-y), h = (w p)(1-p)   (E:2861, E:2873-2874)
__device__ __forceinline__ void grad_hess(double F, int y, double w, double &g, double &h, double &p) {
    double f = fmin(fmax(F, -500.0), 500.0);
    p = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-f)));
    g = __dmul_rn(w, __dsub_rn(p, (double)y));
    h = __dmul_rn(__dmul_rn(w, p), __dsub_rn(1.0, p));
}

// logloss term with p clipped to [1e-15, 1-1e-15]   (E:2320-2325)
__device__ __forceinline__ double loss_term(double p, int y) {
    double pc = fmin(fmax(p, 1e-15), 1.0 - 1e-15);
    return y ? log(pc) : log(__dsub_rn(1.0, pc));
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// data layout: bins column-blocked [nblk][n][16]
// ---------------------------------------------------------------------------

__global__ void k_pack_bins(const uint8_t *__restrict__ src, int64_t rows, int p, int64_t row0,
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
            int lim = counts[f] - 1;
            x = (uint8_t)(c > lim ? lim : c);
        }
        v[k] = x;
    }
    uint4 o;
    memcpy(&o, v, 16);
    reinterpret_cast<uint4 *>(xb)[(int64_t)b * n + row0 + r] = o;
}

__device__ __forceinline__ int bin_of(const uint8_t *__restrict__ xb, int64_t n, int64_t row, int f) {
    return __ldg(xb + (((int64_t)(f >> 4) * n + row) << 4) + (f & 15));
}

// ---------------------------------------------------------------------------
// gradients, F update, loss
// ---------------------------------------------------------------------------

struct TreeDev {         // a pruned tree in the reference's layout
    int n;
    int feat[256];
    int thr[256];
    int left[256];
    int right[256];
    double val[256];
};

__global__ void k_init_grad(const double *__restrict__ F, const uint8_t *__restrict__ y, int64_t n,
                            double w0, double w1, double scale, longlong2 *__restrict__ q) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int yi = y[i];
    double g, h, p;
    grad_hess(F[i], yi, yi ? w1 : w0, g, h, p);
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

// One pass over all rows: traverse the round's tree, F += lr * v (two
// separately rounded operations, like NumPy's F += lr * pred), the loss
// term of the updated F, and the next round's quantised (g, h).
__global__ void __launch_bounds__(kUpdThreads)
k_update(const TreeDev *__restrict__ tree, const uint8_t *__restrict__ xb, int64_t n,
         const uint8_t *__restrict__ y, double w0, double w1, double lr, double scale,
         double *__restrict__ F, longlong2 *__restrict__ q, int32_t *__restrict__ leaf_out,
         double *__restrict__ loss_part) {
    __shared__ int s_feat[256], s_thr[256], s_left[256], s_right[256];
    __shared__ double s_val[256];
    __shared__ double s_red[kUpdThreads / 32];
    int nn = tree->n;
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
            node = (b <= s_thr[node]) ? s_left[node] : s_right[node];
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
}

// Fixed-order sum of the per-block loss partials (deterministic).
__global__ void k_sum_partials(const double *__restrict__ part, int m, double *__restrict__ out) {
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

// ---------------------------------------------------------------------------
// in-bag compaction: mask -> sorted row ids
// ---------------------------------------------------------------------------

constexpr int kCompTile = 4096;

__global__ void k_comp_count(const uint8_t *__restrict__ mask, int64_t n, int32_t *__restrict__ cnt) {
    __shared__ int s[32];
    int64_t base = (int64_t)blockIdx.x * kCompTile;
    int c = 0;
    for (int k = threadIdx.x; k < kCompTile; k += blockDim.x) {
        int64_t i = base + k;
        if (i < n && mask[i]) c++;
    }
    c = warp_sum(c);
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += s[w];
        cnt[blockIdx.x] = t;
    }
}

// Exclusive scan of m ints by one CTA (m is small: tiles of a node or of n).
__global__ void k_scan_small(const int32_t *__restrict__ in, int m, int32_t *__restrict__ out,
                             int32_t *__restrict__ total) {
    __shared__ int32_t s_carry;
    __shared__ int32_t s_w[32];
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    for (int base = 0; base < m; base += blockDim.x) {
        int k = base + threadIdx.x;
        int v = k < m ? in[k] : 0;
        int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        int x = v;
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += t;
        }
        if (lane == 31) s_w[w] = x;
        __syncthreads();
        if (w == 0) {
            int nw = blockDim.x >> 5;
            int y = lane < nw ? s_w[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                int t = __shfl_up_sync(0xffffffffu, y, o);
                if (lane >= o) y += t;
            }
            if (lane < nw) s_w[lane] = y;
        }
        __syncthreads();
        int excl = x - v + (w ? s_w[w - 1] : 0) + s_carry;
        if (k < m) out[k] = excl;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) s_carry = excl + v;
        __syncthreads();
    }
    if (threadIdx.x == 0 && total) *total = s_carry;
}

// Block-wide exclusive scan of one int per thread; returns the block total.
__device__ __forceinline__ int block_excl_scan(int v, int *s_w, int &total) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    if (lane == 31) s_w[w] = x;
    __syncthreads();
    if (w == 0) {
        int y = lane < nw ? s_w[lane] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += t;
        }
        if (lane < nw) s_w[lane] = y;
    }
    __syncthreads();
    int excl = x - v + (w ? s_w[w - 1] : 0);
    total = s_w[nw - 1];
    __syncthreads();
    return excl;
}

__global__ void k_comp_scatter(const uint8_t *__restrict__ mask, int64_t n, const int32_t *__restrict__ off,
                               int32_t *__restrict__ rows) {
    __shared__ int s_w[32];
    int64_t base = (int64_t)blockIdx.x * kCompTile;
    int carry = off[blockIdx.x];
    for (int k0 = 0; k0 < kCompTile; k0 += blockDim.x) {
        int64_t i = base + k0 + threadIdx.x;
        int f = (i < n && mask[i]) ? 1 : 0;
        int tot;
        int e = block_excl_scan(f, s_w, tot);
        if (f) rows[carry + e] = (int32_t)i;
        carry += tot;
    }
}

// ---------------------------------------------------------------------------
// histogram build
// ---------------------------------------------------------------------------

struct HistTask {        // rows d_rows[begin, end) -> staging histogram `stage`
    long long begin, end;
    int stage;
    int left_small;      // wave tasks: the built side is the left child
};

// grid: x = chunk id over all tasks (prefix[ntask] valid chunks), y = feature block
__global__ void __launch_bounds__(kHistThreads)
k_hist(const uint8_t *__restrict__ xb, int64_t n, const int32_t *__restrict__ rows,
       const HistTask *__restrict__ tasks, const int32_t *__restrict__ prefix, int ntask,
       const int32_t *__restrict__ blist, const int16_t *__restrict__ fpos, int nf,
       const longlong2 *__restrict__ q, long long *__restrict__ stage_hist) {
    extern __shared__ unsigned long long sh[];   // [16][256][2]
    __shared__ int s_task;
    int cid = blockIdx.x;
    if (cid >= prefix[ntask]) return;
    if (threadIdx.x == 0) {
        int lo = 0, hi = ntask - 1;
        while (lo < hi) {   // last task with prefix[t] <= cid
            int mid = (lo + hi + 1) >> 1;
            if (prefix[mid] <= cid) lo = mid; else hi = mid - 1;
        }
        s_task = lo;
    }
    for (int k = threadIdx.x; k < kBlk * kBins * 2; k += blockDim.x) sh[k] = 0ull;
    __syncthreads();
    const int t = s_task;
    const HistTask tk = tasks[t];
    const int blk = blist[blockIdx.y];
    long long r0 = tk.begin + (long long)(cid - prefix[t]) * kChunk;
    long long r1 = min(r0 + (long long)kChunk, tk.end);
    unsigned mask = 0;
#pragma unroll
    for (int k = 0; k < kBlk; k++) mask |= (fpos[blk * kBlk + k] >= 0 ? 1u : 0u) << k;
    const uint4 *xv = reinterpret_cast<const uint4 *>(xb) + (int64_t)blk * n;
    for (long long r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
        int row = rows[r];
        uint4 v = __ldg(xv + row);
        longlong2 qq = __ldg(q + row);
        unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < kBlk; k++) {
            if (mask & (1u << k)) {
                int b = (w[k >> 2] >> ((k & 3) * 8)) & 0xff;
                unsigned long long *c = sh + ((k * kBins + b) << 1);
                atomicAdd(c, (unsigned long long)qq.x);
                atomicAdd(c + 1, (unsigned long long)qq.y);
            }
        }
    }
    __syncthreads();
    long long *dst = stage_hist + (int64_t)tk.stage * nf * kBins * kWords;
    for (int idx = threadIdx.x; idx < kBlk * kBins; idx += blockDim.x) {
        int k = idx >> 8, b = idx & 255;
        int jj = fpos[blk * kBlk + k];
        if (jj < 0) continue;
        long long gv = (long long)sh[idx * 2], hv = (long long)sh[idx * 2 + 1];
        long long *o = dst + ((int64_t)jj * kBins + b) * kWords;
        if (gv) {
            atomicAdd((unsigned long long *)(o + 0), (unsigned long long)(gv >> 32));
            atomicAdd((unsigned long long *)(o + 1), (unsigned long long)(gv & 0xffffffffll));
        }
        if (hv) {
            atomicAdd((unsigned long long *)(o + 2), (unsigned long long)(hv >> 32));
            atomicAdd((unsigned long long *)(o + 3), (unsigned long long)(hv & 0xffffffffll));
        }
    }
}

// ---------------------------------------------------------------------------
// partition (stable) of wave nodes
// ---------------------------------------------------------------------------

struct PartTask {
    long long begin, end;   // segment of d_rows
    int feat, thr;          // split: bin(feat) <= thr goes left
    int tile0;              // first tile id of this task
    int ntile;
};

__device__ __forceinline__ int find_task_by_tile(const PartTask *tasks, int ntask, int tile) {
    int lo = 0, hi = ntask - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (tasks[mid].tile0 <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__global__ void __launch_bounds__(kPartThreads)
k_part_count(const uint8_t *__restrict__ xb, int64_t n, const int32_t *__restrict__ rows,
             const PartTask *__restrict__ tasks, int ntask, int32_t *__restrict__ tile_cnt) {
    __shared__ int s[32];
    int tile = blockIdx.x;
    int t = find_task_by_tile(tasks, ntask, tile);
    PartTask tk = tasks[t];
    long long r0 = tk.begin + (long long)(tile - tk.tile0) * kPartTile;
    long long r1 = min(r0 + kPartTile, tk.end);
    int c = 0;
    for (long long r = r0 + threadIdx.x; r < r1; r += blockDim.x)
        c += bin_of(xb, n, rows[r], tk.feat) <= tk.thr;
    c = warp_sum(c);
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int tot = 0;
        for (int w = 0; w < kPartThreads / 32; w++) tot += s[w];
        tile_cnt[tile] = tot;
    }
}

// One CTA per task: exclusive scan of its tiles' left counts; n_left.
__global__ void k_part_scan(const PartTask *__restrict__ tasks, const int32_t *__restrict__ tile_cnt,
                            int32_t *__restrict__ tile_off, long long *__restrict__ n_left) {
    __shared__ int s_w[32];
    __shared__ int s_carry;
    PartTask tk = tasks[blockIdx.x];
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    for (int b = 0; b < tk.ntile; b += blockDim.x) {
        int k = b + threadIdx.x;
        int v = k < tk.ntile ? tile_cnt[tk.tile0 + k] : 0;
        int tot;
        int e = block_excl_scan(v, s_w, tot);
        if (k < tk.ntile) tile_off[tk.tile0 + k] = s_carry + e;
        __syncthreads();
        if (threadIdx.x == 0) s_carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) n_left[blockIdx.x] = s_carry;
}

__global__ void __launch_bounds__(kPartThreads)
k_part_scatter(const uint8_t *__restrict__ xb, int64_t n, const int32_t *__restrict__ rows,
               const PartTask *__restrict__ tasks, int ntask, const int32_t *__restrict__ tile_off,
               const long long *__restrict__ n_left, int32_t *__restrict__ tmp) {
    __shared__ int s_w[32];
    int tile = blockIdx.x;
    int t = find_task_by_tile(tasks, ntask, tile);
    PartTask tk = tasks[t];
    long long tstart = tk.begin + (long long)(tile - tk.tile0) * kPartTile;
    long long r1 = min(tstart + kPartTile, tk.end);
    long long nl = n_left[t];
    long long lcar = tile_off[tile];                         // lefts before this tile
    long long rcar = (tstart - tk.begin) - lcar;             // rights before this tile
    for (long long r0 = tstart; r0 < r1; r0 += blockDim.x) {
        long long r = r0 + threadIdx.x;
        int row = 0, f = 0;
        bool in = r < r1;
        if (in) {
            row = rows[r];
            f = bin_of(xb, n, row, tk.feat) <= tk.thr;
        }
        int tot;
        int e = block_excl_scan(f, s_w, tot);
        if (in) {
            int pos_in_chunk = (int)(r - r0);
            if (f) tmp[tk.begin + lcar + e] = row;
            else tmp[tk.begin + nl + rcar + (pos_in_chunk - e)] = row;
        }
        int cnt = (int)min((long long)blockDim.x, r1 - r0);
        lcar += tot;
        rcar += cnt - tot;
    }
}

__global__ void k_part_copyback(const PartTask *__restrict__ tasks, int ntask, const int32_t *__restrict__ tmp,
                                int32_t *__restrict__ rows) {
    int tile = blockIdx.x;
    int t = find_task_by_tile(tasks, ntask, tile);
    PartTask tk = tasks[t];
    long long r0 = tk.begin + (long long)(tile - tk.tile0) * kPartTile;
    long long r1 = min(r0 + kPartTile, tk.end);
    for (long long r = r0 + threadIdx.x; r < r1; r += blockDim.x) rows[r] = tmp[r];
}

// ---------------------------------------------------------------------------
// wave planning, sibling subtraction
// ---------------------------------------------------------------------------

struct WaveNode {
    long long begin, end;
    int parent_slot, left_slot, right_slot;
    int pad;
    long long gtotal;      // rows of the node over all ranks
};

// After the partition: the smaller side becomes a histogram task into
// staging index k; child row counts for the split kernel.
// `n_left` are this rank's counts (they place the rows), `gl`/`gtot` the
// counts over all ranks (they pick the smaller side, E:701-709, the same on
// every rank).
__global__ void k_plan(const WaveNode *__restrict__ wn, int w, const long long *__restrict__ n_left,
                       const long long *__restrict__ gl, const long long *__restrict__ gtot,
                       HistTask *__restrict__ ht, int32_t *__restrict__ prefix,
                       long long *__restrict__ child_n) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int acc = 0;
    for (int k = 0; k < w; k++) {
        long long nl = n_left[k];
        long long gnl = gl[k], gnr = gtot[k] - gl[k];
        bool left_small = gnl <= gnr;
        HistTask t;
        t.begin = left_small ? wn[k].begin : wn[k].begin + nl;
        t.end = left_small ? wn[k].begin + nl : wn[k].end;
        t.stage = k;
        t.left_small = left_small ? 1 : 0;
        ht[k] = t;
        prefix[k] = acc;
        acc += (int)((t.end - t.begin + kChunk - 1) / kChunk);
        child_n[2 * k] = gnl;
        child_n[2 * k + 1] = gnr;
    }
    prefix[w] = acc;
}

// small side <- staging[k]; large side <- parent - staging[k]
__global__ void k_finish(const WaveNode *__restrict__ wn, const HistTask *__restrict__ ht,
                         const long long *__restrict__ stage, long long *__restrict__ pool, int64_t words) {
    int k = blockIdx.y;
    WaveNode nd = wn[k];
    bool left_small = ht[k].left_small != 0;
    int ss = left_small ? nd.left_slot : nd.right_slot;
    int ls = left_small ? nd.right_slot : nd.left_slot;
    const long long *st = stage + (int64_t)k * words;
    const long long *par = pool + (int64_t)nd.parent_slot * words;
    long long *sm = pool + (int64_t)ss * words;
    long long *lg = pool + (int64_t)ls * words;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words;
         i += (int64_t)gridDim.x * blockDim.x) {
        long long v = st[i];
        sm[i] = v;
        lg[i] = par[i] - v;
    }
}

__global__ void k_copy_stage(const long long *__restrict__ stage, long long *__restrict__ dst, int64_t words) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = stage[i];
}

__global__ void k_zero(long long *__restrict__ p, int64_t words) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words;
         i += (int64_t)gridDim.x * blockDim.x)
        p[i] = 0;
}

// ---------------------------------------------------------------------------
// split finder
// ---------------------------------------------------------------------------

struct SplitTask {
    int slot;
    int eval;              // host-side condition (depth); device adds n/H checks
    long long n;           // rows (global) of the node, or -1 = read child_n[cidx]
    int cidx;
    int pad;
};

struct SplitOut {
    double G, H;           // exact totals, rounded once
    double gain;
    long long n;
    int feat;              // original feature id, -1 = no split
    int bin;
};

struct Best {
    double gain;
    int jj, bin;
};

__device__ __forceinline__ bool better(const Best &a, const Best &b) {   // a beats b
    if (a.jj < 0) return false;
    if (b.jj < 0) return true;
    if (a.gain > b.gain) return true;
    if (b.gain > a.gain) return false;
    if (a.jj != b.jj) return a.jj < b.jj;
    return a.bin < b.bin;
}

__device__ __forceinline__ i128 shfl_up_i128(i128 v, int o) {
    long long lo = (long long)(unsigned long long)v;
    long long hi = (long long)(v >> 64);
    lo = __shfl_up_sync(0xffffffffu, lo, o);
    hi = __shfl_up_sync(0xffffffffu, hi, o);
    return ((i128)hi << 64) | (i128)(unsigned long long)lo;
}

__device__ __forceinline__ i128 shfl_i128(i128 v, int src) {
    long long lo = (long long)(unsigned long long)v;
    long long hi = (long long)(v >> 64);
    lo = __shfl_sync(0xffffffffu, lo, src);
    hi = __shfl_sync(0xffffffffu, hi, src);
    return ((i128)hi << 64) | (i128)(unsigned long long)lo;
}

// One CTA per node; warp w scans features jj = w, w+8, ...; lane l owns bins 8l..8l+7.
__global__ void __launch_bounds__(kSplitThreads)
k_split(const SplitTask *__restrict__ tasks, const long long *__restrict__ child_n,
        const long long *__restrict__ pool, int nf, const int32_t *__restrict__ fidx,
        const int32_t *__restrict__ counts, int S, double lam, double mcw, long long msl,
        SplitOut *__restrict__ out) {
    __shared__ Best s_best[kSplitThreads / 32];
    __shared__ double s_GH[2];
    const SplitTask tk = tasks[blockIdx.x];
    const long long *hist = pool + (int64_t)tk.slot * nf * kBins * kWords;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const double sc = pow2(-S);
    long long nrows = tk.n >= 0 ? tk.n : child_n[tk.cidx];

    // node totals from feature position 0 (every row lands in exactly one bin)
    if (warp == 0) {
        i128 tg = 0, th = 0;
        for (int b = lane; b < kBins; b += 32) {
            const long long *c = hist + (int64_t)b * kWords;
            tg += cell(c[0], c[1]);
            th += cell(c[2], c[3]);
        }
        for (int o = 16; o > 0; o >>= 1) {
            tg += shfl_i128(tg, lane ^ o);   // butterfly: all lanes get the sum
            th += shfl_i128(th, lane ^ o);
        }
        if (lane == 0) {
            s_GH[0] = __dmul_rn(i128_to_double(tg), sc);
            s_GH[1] = __dmul_rn(i128_to_double(th), sc);
        }
    }
    __syncthreads();
    const double Gt = s_GH[0], Ht = s_GH[1];
    const bool can = tk.eval && nrows >= msl && Ht >= mcw;
    Best best = {-1e9, -1, 0};
    if (can) {
        const double parent = __ddiv_rn(__dmul_rn(Gt, Gt), __dadd_rn(Ht, lam));
        for (int jj = warp; jj < nf; jj += kSplitThreads / 32) {
            int nb = counts[fidx[jj]];
            if (nb < 2) continue;
            const long long *hf = hist + (int64_t)jj * kBins * kWords;
            i128 g[8], h[8];
            i128 lg = 0, lh = 0, tg_f = 0, th_f = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const longlong2 *c = reinterpret_cast<const longlong2 *>(hf + (int64_t)(lane * 8 + k) * kWords);
                longlong2 a = c[0], b = c[1];
                g[k] = cell(a.x, a.y);
                h[k] = cell(b.x, b.y);
                lg += g[k];
                lh += h[k];
            }
            // exclusive prefix of lane totals
            i128 xg = lg, xh = lh;
            for (int o = 1; o < 32; o <<= 1) {
                i128 tg2 = shfl_up_i128(xg, o), th2 = shfl_up_i128(xh, o);
                if (lane >= o) { xg += tg2; xh += th2; }
            }
            tg_f = shfl_i128(xg, 31);
            th_f = shfl_i128(xh, 31);
            i128 pg = xg - lg, ph = xh - lh;
            Best lb = {-1e9, -1, 0};
#pragma unroll
            for (int k = 0; k < 8; k++) {
                int b = lane * 8 + k;
                pg += g[k];
                ph += h[k];
                if (b <= nb - 2) {
                    double GL = __dmul_rn(i128_to_double(pg), sc);
                    double HL = __dmul_rn(i128_to_double(ph), sc);
                    double GR = __dmul_rn(i128_to_double(tg_f - pg), sc);
                    double HR = __dmul_rn(i128_to_double(th_f - ph), sc);
                    if (!(HL < mcw || HR < mcw)) {
                        double gain = __dsub_rn(
                            __dadd_rn(__ddiv_rn(__dmul_rn(GL, GL), __dadd_rn(HL, lam)),
                                      __ddiv_rn(__dmul_rn(GR, GR), __dadd_rn(HR, lam))),
                            parent);
                        if (gain > lb.gain) { lb.gain = gain; lb.jj = jj; lb.bin = b; }
                    }
                }
            }
            for (int o = 16; o > 0; o >>= 1) {
                Best ob;
                ob.gain = __shfl_xor_sync(0xffffffffu, lb.gain, o);
                ob.jj = __shfl_xor_sync(0xffffffffu, lb.jj, o);
                ob.bin = __shfl_xor_sync(0xffffffffu, lb.bin, o);
                if (better(ob, lb)) lb = ob;
            }
            if (better(lb, best)) best = lb;
        }
    }
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        Best b = s_best[0];
        for (int w = 1; w < kSplitThreads / 32; w++)
            if (better(s_best[w], b)) b = s_best[w];
        SplitOut o;
        o.G = Gt;
        o.H = Ht;
        o.n = nrows;
        o.gain = b.gain;
        o.feat = b.jj >= 0 ? fidx[b.jj] : -1;
        o.bin = b.bin;
        out[blockIdx.x] = o;
    }
}

// ---------------------------------------------------------------------------
// predict (ensemble traversal, E:863-884)
// ---------------------------------------------------------------------------

struct PNode {          // 8 bytes per node
    int16_t feat;       // -1 = leaf
    uint8_t thr;
    uint8_t pad;
    int16_t left, right;// tree-local ids
};

__global__ void __launch_bounds__(256)
k_predict(const uint8_t *__restrict__ xr, int64_t n, int p, const PNode *__restrict__ nodes,
          const double *__restrict__ vals, const int32_t *__restrict__ off, int ntree, double lr,
          double base, double *__restrict__ F, double *__restrict__ proba) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t *row = xr + i * p;
    double acc = 0.0;
    for (int t = 0; t < ntree; t++) {
        int o = __ldg(off + t);
        int node = 0;
        PNode nd = nodes[o];
        while (nd.feat >= 0) {
            int b = __ldg(row + nd.feat);
            node = b <= nd.thr ? nd.left : nd.right;
            nd = nodes[o + node];
        }
        acc = __dadd_rn(acc, __dmul_rn(lr, __ldg(vals + o + node)));
    }
    double f = __dadd_rn(acc, base);
    if (F) F[i] = f;
    if (proba) {
        double c = fmin(fmax(f, -500.0), 500.0);
        proba[i] = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-c)));
    }
}

}  // namespace

// ===========================================================================
// host side
// ===========================================================================

struct gbm_ctx {
    int dev = -1;
    cudaStream_t st = nullptr;
    std::string err;
    gbm_comm *comm = nullptr;
    int timeout_ms = 60000;

    // data
    int64_t n = 0;          // local rows
    int64_t n_global = 0;
    int32_t p = 0, nblk = 0;
    uint8_t *d_xb = nullptr;
    int32_t *d_counts = nullptr;
    std::vector<int32_t> counts;
    uint8_t *d_y = nullptr;
    double *d_F = nullptr;
    longlong2 *d_q = nullptr;
    double w[2] = {1.0, 1.0};
    double base = 0.0;
    int S = 0;
    bool have_bins = false, have_labels = false;

    // round buffers
    uint8_t *d_mask = nullptr;
    int32_t *d_rows = nullptr, *d_tmp = nullptr;
    int32_t *d_cnt = nullptr, *d_off = nullptr, *d_total = nullptr;
    int32_t *d_blist = nullptr, *d_fidx = nullptr;
    int16_t *d_fpos = nullptr;
    int nf_cap = 0;
    long long *d_pool = nullptr;
    int pool_slots = 0;
    long long *d_stage = nullptr;
    int stage_slots = 0;
    int64_t slot_words = 0;
    HistTask *d_htask = nullptr;
    int32_t *d_hprefix = nullptr;
    PartTask *d_ptask = nullptr;
    int32_t *d_tile_cnt = nullptr, *d_tile_off = nullptr;
    int tile_cap = 0;
    long long *d_nleft = nullptr, *d_nleft_g = nullptr, *d_gtot = nullptr, *d_child_n = nullptr;
    long long *d_count = nullptr;
    WaveNode *d_wave = nullptr;
    SplitTask *d_stask = nullptr;
    SplitOut *d_sout = nullptr;
    TreeDev *d_tree = nullptr;
    int32_t *d_leaf = nullptr;
    double *d_loss_part = nullptr, *d_loss = nullptr;
    int upd_blocks = 0;
    // pinned host mirrors
    SplitOut *h_sout = nullptr;
    long long *h_nleft = nullptr, *h_nloc = nullptr, *h_count = nullptr;
    double *h_loss = nullptr;
    int32_t *h_total = nullptr;
    uint8_t *h_mask = nullptr;

    // predict
    uint8_t *d_px = nullptr;
    int64_t pn = 0, pn_cap = 0;
    int32_t pp = 0;
    PNode *d_pnodes = nullptr;
    double *d_pvals = nullptr;
    int32_t *d_poff = nullptr;
    int32_t p_ntree = 0;
    int64_t p_nodes_cap = 0;
    int32_t p_trees_cap = 0;
    int32_t p_nfeat = 0;
    double *d_pF = nullptr, *d_pP = nullptr;

    // instrumentation
    long long launches = 0;          // every kernel this context launched
    bool profiling = false;
    long long hist_launches = 0, hist_rows = 0, waves = 0;
    double hist_ms = 0.0, alg_bytes = 0.0;
    std::vector<cudaEvent_t> hist_ev;  // pairs recorded around k_hist launches
    int hist_ev_used = 0;
    cudaEvent_t mark[16] = {};
};

namespace {

int fail(gbm_ctx *c, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c) c->err = buf;
    return code;
}

#define CK(call)                                                                          \
    do {                                                                                  \
        cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess)                                                            \
            return fail(ctx, GBM_ERR_CUDA, "%s failed: %s (%s:%d)", #call,                \
                        cudaGetErrorString(e_), __FILE__, __LINE__);                      \
    } while (0)

#define CKL()                                                                             \
    do {                                                                                  \
        ctx->launches++;                                                                  \
        cudaError_t e_ = cudaGetLastError();                                              \
        if (e_ != cudaSuccess)                                                            \
            return fail(ctx, GBM_ERR_CUDA, "kernel launch failed: %s (%s:%d)",            \
                        cudaGetErrorString(e_), __FILE__, __LINE__);                      \
    } while (0)

#define TRY(x)                      \
    do {                            \
        int r_ = (x);               \
        if (r_ != GBM_OK) return r_;\
    } while (0)

template <typename T>
int dalloc(gbm_ctx *ctx, T **p, size_t count) {
    if (*p) { cudaFree(*p); *p = nullptr; }
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc((void **)p, count * sizeof(T));
    if (e != cudaSuccess)
        return fail(ctx, GBM_ERR_ALLOC, "cudaMalloc(%zu bytes) failed: %s", count * sizeof(T),
                    cudaGetErrorString(e));
    return GBM_OK;
}

template <typename T>
int halloc(gbm_ctx *ctx, T **p, size_t count) {
    if (*p) { cudaFreeHost(*p); *p = nullptr; }
    if (count == 0) count = 1;
    cudaError_t e = cudaMallocHost((void **)p, count * sizeof(T));
    if (e != cudaSuccess)
        return fail(ctx, GBM_ERR_ALLOC, "cudaMallocHost(%zu bytes) failed: %s", count * sizeof(T),
                    cudaGetErrorString(e));
    return GBM_OK;
}

int grid_for(int64_t work, int threads, int cap = 1 << 30) {
    int64_t g = (work + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (int)g;
}

// S such that kChunk rows of |g| <= wmax (h <= wmax/4) never overflow int64.
int scale_bits_for(double wmax) {
    double m = std::max(1.0, wmax);
    int need = (int)std::ceil(std::log2((double)kChunk * m));
    return 62 - need;
}

int sync_stream(gbm_ctx *ctx) {
    if (ctx->comm) return gbm_comm_sync(ctx->comm, ctx->st, ctx->timeout_ms, ctx->err);
    CK(cudaStreamSynchronize(ctx->st));
    return GBM_OK;
}

// ---- per-round feature tables ---------------------------------------------

struct RoundFeat {
    int nf;
    std::vector<int32_t> blist;
    std::vector<int16_t> fpos;
};

int setup_features(gbm_ctx *ctx, const int32_t *fidx, int nf, RoundFeat &rf) {
    rf.nf = nf;
    rf.fpos.assign((size_t)ctx->nblk * kBlk, (int16_t)-1);
    for (int jj = 0; jj < nf; jj++) {
        int f = fidx[jj];
        if (f < 0 || f >= ctx->p) return fail(ctx, GBM_ERR_ARG, "feat_idx[%d]=%d out of range", jj, f);
        if (jj > 0 && fidx[jj - 1] >= f) return fail(ctx, GBM_ERR_ARG, "feat_idx must be strictly increasing");
        rf.fpos[(size_t)f] = (int16_t)jj;
    }
    rf.blist.clear();
    for (int b = 0; b < ctx->nblk; b++) {
        bool any = false;
        for (int k = 0; k < kBlk; k++) any |= rf.fpos[(size_t)b * kBlk + k] >= 0;
        if (any) rf.blist.push_back(b);
    }
    CK(cudaMemcpyAsync(ctx->d_fidx, fidx, sizeof(int32_t) * nf, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_fpos, rf.fpos.data(), sizeof(int16_t) * rf.fpos.size(), cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_blist, rf.blist.data(), sizeof(int32_t) * rf.blist.size(), cudaMemcpyHostToDevice, ctx->st));
    return GBM_OK;
}

int ensure_round_buffers(gbm_ctx *ctx, int nf, int max_leaves) {
    int need_nf = std::max(nf, 1);
    int slots = 4 * max_leaves + 8;
    int stage = std::min(kMaxWave, 2 * max_leaves + 2);
    if (need_nf > ctx->nf_cap || slots > ctx->pool_slots || stage > ctx->stage_slots) {
        ctx->nf_cap = std::max(need_nf, ctx->nf_cap);
        ctx->pool_slots = std::max(slots, ctx->pool_slots);
        ctx->stage_slots = std::max(stage, ctx->stage_slots);
        ctx->slot_words = (int64_t)ctx->nf_cap * kBins * kWords;
        TRY(dalloc(ctx, &ctx->d_pool, (size_t)ctx->pool_slots * ctx->slot_words));
        TRY(dalloc(ctx, &ctx->d_stage, (size_t)ctx->stage_slots * ctx->slot_words));
        TRY(dalloc(ctx, &ctx->d_fidx, (size_t)ctx->nf_cap));
    }
    return GBM_OK;
}

// ---- device work of one wave ------------------------------------------------

struct WaveIn {
    long long gtotal;      // rows over all ranks
    long long begin, end;  // this rank's segment
    int feat, thr;
    int parent_slot, left_slot, right_slot;
    int depth_ok;          // children may split (depth + 1 < max_depth)
};

struct ChildRes {
    double G, H, gain;
    long long n;
    int feat, bin;
};

int launch_split(gbm_ctx *ctx, const RoundFeat &rf, const std::vector<SplitTask> &tasks,
                 const gbm_params *P) {
    CK(cudaMemcpyAsync(ctx->d_stask, tasks.data(), sizeof(SplitTask) * tasks.size(),
                       cudaMemcpyHostToDevice, ctx->st));
    k_split<<<(unsigned)tasks.size(), kSplitThreads, 0, ctx->st>>>(
        ctx->d_stask, ctx->d_child_n, ctx->d_pool, rf.nf, ctx->d_fidx, ctx->d_counts, ctx->S,
        P->reg_lambda, P->min_child_weight, (long long)P->min_samples_leaf, ctx->d_sout);
    CKL();
    return GBM_OK;
}

int launch_hist(gbm_ctx *ctx, const RoundFeat &rf, int ntask, int max_chunks) {
    if (max_chunks <= 0) return GBM_OK;
    dim3 grid((unsigned)max_chunks, (unsigned)rf.blist.size());
    size_t smem = (size_t)kBlk * kBins * 2 * sizeof(unsigned long long);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->profiling) {
        if ((int)ctx->hist_ev.size() < ctx->hist_ev_used + 2) {
            for (int k = 0; k < 2; k++) {
                cudaEvent_t e;
                CK(cudaEventCreate(&e));
                ctx->hist_ev.push_back(e);
            }
        }
        e0 = ctx->hist_ev[ctx->hist_ev_used];
        e1 = ctx->hist_ev[ctx->hist_ev_used + 1];
        ctx->hist_ev_used += 2;
        CK(cudaEventRecord(e0, ctx->st));
    }
    k_hist<<<grid, kHistThreads, smem, ctx->st>>>(ctx->d_xb, ctx->n, ctx->d_rows, ctx->d_htask,
                                                   ctx->d_hprefix, ntask, ctx->d_blist, ctx->d_fpos,
                                                   rf.nf, ctx->d_q, ctx->d_stage);
    CKL();
    if (ctx->profiling) CK(cudaEventRecord(e1, ctx->st));
    ctx->hist_launches++;
    return GBM_OK;
}

// Fold the k_hist event pairs of the last wave into the totals (after a sync).
int collect_hist_events(gbm_ctx *ctx) {
    for (int k = 0; k + 1 < ctx->hist_ev_used; k += 2) {
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, ctx->hist_ev[k], ctx->hist_ev[k + 1]));
        ctx->hist_ms += ms;
    }
    ctx->hist_ev_used = 0;
    return GBM_OK;
}

// Root: histogram of all in-bag rows into `slot`, then its split.
int device_root(gbm_ctx *ctx, const RoundFeat &rf, long long n_sub, long long n_sub_g, int slot, int eval,
                const gbm_params *P, ChildRes &res) {
    int64_t words = (int64_t)rf.nf * kBins * kWords;
    k_zero<<<grid_for(words, 256, 4096), 256, 0, ctx->st>>>(ctx->d_stage, words);
    CKL();
    HistTask ht{0, n_sub, 0, 1};
    int chunks = (int)((n_sub + kChunk - 1) / kChunk);
    int32_t pre[2] = {0, chunks};
    CK(cudaMemcpyAsync(ctx->d_htask, &ht, sizeof ht, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_hprefix, pre, sizeof pre, cudaMemcpyHostToDevice, ctx->st));
    TRY(launch_hist(ctx, rf, 1, chunks));
    if (ctx->comm) TRY(gbm_comm_allreduce_i64(ctx->comm, ctx->d_stage, words, ctx->st, ctx->timeout_ms, ctx->err));
    // stage slot 0 -> pool slot (words of the selected features are contiguous)
    k_copy_stage<<<grid_for(words, 256, 4096), 256, 0, ctx->st>>>(ctx->d_stage,
                                                                   ctx->d_pool + (int64_t)slot * words, words);
    CKL();
    std::vector<SplitTask> st(1);
    st[0] = SplitTask{slot, eval, n_sub_g, 0, 0};
    TRY(launch_split(ctx, rf, st, P));
    CK(cudaMemcpyAsync(ctx->h_sout, ctx->d_sout, sizeof(SplitOut), cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    if (ctx->profiling) TRY(collect_hist_events(ctx));
    ctx->hist_rows += n_sub;
    ctx->alg_bytes += (double)n_sub_g * (rf.nf + 8);
    const SplitOut &o = ctx->h_sout[0];
    res = ChildRes{o.G, o.H, o.gain, o.n, o.feat, o.bin};
    return GBM_OK;
}

// Expand a wave of nodes: partition, smaller-child histogram, subtraction,
// children's splits.  Fills nl[k] and kids[2k] (left), kids[2k+1] (right).
int device_wave(gbm_ctx *ctx, const RoundFeat &rf, const std::vector<WaveIn> &win,
                const gbm_params *P, std::vector<long long> &nl, std::vector<ChildRes> &kids) {
    int w = (int)win.size();
    int64_t words = (int64_t)rf.nf * kBins * kWords;
    // partition tasks
    std::vector<PartTask> pt(w);
    std::vector<WaveNode> wn(w);
    int tiles = 0, max_chunks = 0;
    for (int k = 0; k < w; k++) {
        long long sz = win[k].end - win[k].begin;
        int nt = (int)((sz + kPartTile - 1) / kPartTile);
        if (nt < 1) nt = 1;
        pt[k] = PartTask{win[k].begin, win[k].end, win[k].feat, win[k].thr, tiles, nt};
        tiles += nt;
        wn[k] = WaveNode{win[k].begin, win[k].end, win[k].parent_slot, win[k].left_slot,
                         win[k].right_slot, 0, win[k].gtotal};
        max_chunks += (int)((sz / 2 + kChunk - 1) / kChunk);
    }
    if (ctx->comm) {
        // the globally smaller side may be the locally larger one
        max_chunks = 0;
        for (int k = 0; k < w; k++)
            max_chunks += (int)((win[k].end - win[k].begin + kChunk - 1) / kChunk);
    }
    if (tiles > ctx->tile_cap) {
        ctx->tile_cap = tiles * 2;
        TRY(dalloc(ctx, &ctx->d_tile_cnt, (size_t)ctx->tile_cap));
        TRY(dalloc(ctx, &ctx->d_tile_off, (size_t)ctx->tile_cap));
    }
    CK(cudaMemcpyAsync(ctx->d_ptask, pt.data(), sizeof(PartTask) * w, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_wave, wn.data(), sizeof(WaveNode) * w, cudaMemcpyHostToDevice, ctx->st));
    k_part_count<<<tiles, kPartThreads, 0, ctx->st>>>(ctx->d_xb, ctx->n, ctx->d_rows, ctx->d_ptask, w,
                                                      ctx->d_tile_cnt);
    CKL();
    k_part_scan<<<w, 256, 0, ctx->st>>>(ctx->d_ptask, ctx->d_tile_cnt, ctx->d_tile_off, ctx->d_nleft);
    CKL();
    k_part_scatter<<<tiles, kPartThreads, 0, ctx->st>>>(ctx->d_xb, ctx->n, ctx->d_rows, ctx->d_ptask, w,
                                                        ctx->d_tile_off, ctx->d_nleft, ctx->d_tmp);
    CKL();
    k_part_copyback<<<tiles, kPartThreads, 0, ctx->st>>>(ctx->d_ptask, w, ctx->d_tmp, ctx->d_rows);
    CKL();
    {
        // local n_left places the rows; counts summed over ranks pick the
        // smaller side and feed the min_samples_leaf checks.
        std::vector<long long> gt(w);
        for (int k = 0; k < w; k++) gt[k] = win[k].gtotal;
        CK(cudaMemcpyAsync(ctx->d_gtot, gt.data(), sizeof(long long) * w, cudaMemcpyHostToDevice, ctx->st));
        const long long *gl = ctx->d_nleft;
        if (ctx->comm) {
            CK(cudaMemcpyAsync(ctx->d_nleft_g, ctx->d_nleft, sizeof(long long) * w, cudaMemcpyDeviceToDevice,
                               ctx->st));
            TRY(gbm_comm_allreduce_i64(ctx->comm, ctx->d_nleft_g, w, ctx->st, ctx->timeout_ms, ctx->err));
            gl = ctx->d_nleft_g;
        }
        k_plan<<<1, 32, 0, ctx->st>>>(ctx->d_wave, w, ctx->d_nleft, gl, ctx->d_gtot, ctx->d_htask,
                                      ctx->d_hprefix, ctx->d_child_n);
        CKL();
    }
    k_zero<<<grid_for(words * w, 256, 8192), 256, 0, ctx->st>>>(ctx->d_stage, words * w);
    CKL();
    TRY(launch_hist(ctx, rf, w, max_chunks));
    if (ctx->comm)
        TRY(gbm_comm_allreduce_i64(ctx->comm, ctx->d_stage, words * w, ctx->st, ctx->timeout_ms, ctx->err));
    {
        dim3 g((unsigned)grid_for(words, 256, 64), (unsigned)w);
        k_finish<<<g, 256, 0, ctx->st>>>(ctx->d_wave, ctx->d_htask, ctx->d_stage, ctx->d_pool, words);
        CKL();
    }
    std::vector<SplitTask> st(2 * w);
    for (int k = 0; k < w; k++) {
        st[2 * k] = SplitTask{win[k].left_slot, win[k].depth_ok, -1, 2 * k, 0};
        st[2 * k + 1] = SplitTask{win[k].right_slot, win[k].depth_ok, -1, 2 * k + 1, 0};
    }
    TRY(launch_split(ctx, rf, st, P));
    CK(cudaMemcpyAsync(ctx->h_sout, ctx->d_sout, sizeof(SplitOut) * 2 * w, cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaMemcpyAsync(ctx->h_nleft, ctx->d_child_n, sizeof(long long) * 2 * w, cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaMemcpyAsync(ctx->h_nloc, ctx->d_nleft, sizeof(long long) * w, cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    if (ctx->profiling) TRY(collect_hist_events(ctx));
    ctx->waves++;
    nl.resize(w);
    kids.resize(2 * w);
    for (int k = 0; k < w; k++) {
        nl[k] = ctx->h_nloc[k];
        long long tot = win[k].end - win[k].begin;
        ctx->hist_rows += std::min(nl[k], tot - nl[k]);   // local rows of the built side (approx. with comm)
        for (int s = 0; s < 2; s++) {
            const SplitOut &o = ctx->h_sout[2 * k + s];
            kids[2 * k + s] = ChildRes{o.G, o.H, o.gain, o.n, o.feat, o.bin};
        }
    }
    return GBM_OK;
}

// ---- slot pool ----------------------------------------------------------------

struct SlotPool {
    std::vector<int> free_;
    void reset(int n) {
        free_.clear();
        for (int i = n - 1; i >= 0; i--) free_.push_back(i);
    }
    int take() {
        if (free_.empty()) return -1;
        int s = free_.back();
        free_.pop_back();
        return s;
    }
    void give(int s) {
        if (s >= 0) free_.push_back(s);
    }
    int avail() const { return (int)free_.size(); }
};

// ---- tree output helpers --------------------------------------------------------

struct HostTree {
    std::vector<int32_t> tf, tl, tr;
    std::vector<int64_t> tt;
    std::vector<double> tv, sg;
    int nc = 0;
    void init(int m) {
        tf.assign(m, -1); tl.assign(m, -1); tr.assign(m, -1);
        tt.assign(m, 0); tv.assign(m, 0.0); sg.assign(m, 0.0);
        nc = 0;
    }
};

// ---- best-first replay (E:517-823) ------------------------------------------------

struct Cand {
    int node = 0, depth = 0, feat = -1, bin = 0;
    double gain = -1.0, val = 0.0;
    bool active = false;
    // device state
    int dslot = -1;
    long long begin = 0, end = 0;   // this rank's rows
    long long gtotal = 0;           // rows over all ranks
    // expansion results
    int expanded = 0;
    long long nl = 0, nr = 0;
    ChildRes kid[2];
    int kslot[2] = {-1, -1};
};

int build_leafwise(gbm_ctx *ctx, const RoundFeat &rf, long long n_sub, long long n_sub_g,
                   const gbm_params *P, HostTree &T) {
    const int max_leaves = P->max_leaves;
    const int MAXC = max_leaves + 2;
    const double lam = P->reg_lambda, mcw = P->min_child_weight, gamma = P->gamma;
    const long long msl = P->min_samples_leaf;
    T.init(2 * max_leaves + 2);
    SlotPool pool;
    pool.reset(ctx->pool_slots);
    int node_count = 0;
    int root = node_count++;
    int s0 = pool.take();
    ChildRes r;
    TRY(device_root(ctx, rf, n_sub, n_sub_g, s0, 1, P, r));
    double root_val = -r.G / (r.H + lam);
    if (n_sub_g < msl || r.H < mcw) {
        T.tf[root] = -1; T.tv[root] = root_val; T.nc = node_count;
        return GBM_OK;
    }
    std::vector<Cand> c(MAXC);
    c[0].node = root; c[0].depth = 0; c[0].gain = r.feat >= 0 ? r.gain : -1.0;
    c[0].feat = r.feat; c[0].bin = r.bin; c[0].val = root_val; c[0].active = true;
    c[0].dslot = s0; c[0].begin = 0; c[0].end = n_sub; c[0].gtotal = n_sub_g;
    if (r.feat < 0) {
        T.tf[root] = -1; T.tv[root] = root_val; T.nc = node_count;
        return GBM_OK;
    }
    int n_splits = 0;
    std::vector<long long> nl;
    std::vector<ChildRes> kids;
    while (n_splits < max_leaves - 1) {
        int ci = -1;
        double bg = gamma;
        for (int s = 0; s < MAXC; s++)
            if (c[s].active && c[s].feat >= 0 && c[s].gain > bg) { bg = c[s].gain; ci = s; }
        if (ci < 0) break;
        if (!c[ci].expanded) {
            // Wave: the best unexpanded candidates in selection order.
            std::vector<int> order;
            for (int s = 0; s < MAXC; s++)
                if (c[s].active && c[s].feat >= 0 && c[s].gain > gamma && !c[s].expanded) order.push_back(s);
            std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return c[a].gain > c[b].gain; });
            int budget = std::min<int>((int)order.size(), max_leaves - 1 - n_splits);
            budget = std::min(budget, std::min(kMaxWave, ctx->stage_slots));
            if (pool.avail() < 2 * budget) {
                // reclaim children of expanded candidates that were never applied
                for (int s = 0; s < MAXC; s++)
                    if (c[s].active && c[s].expanded) {
                        pool.give(c[s].kslot[0]); pool.give(c[s].kslot[1]);
                        c[s].kslot[0] = c[s].kslot[1] = -1;
                        c[s].expanded = 0;
                    }
                budget = std::min(budget, pool.avail() / 2);
            }
            if (budget < 1) return fail(ctx, GBM_ERR_STATE, "histogram slot pool exhausted");
            // ci is first in `order` (largest gain, lowest slot)
            std::vector<WaveIn> win;
            std::vector<int> who;
            for (int q = 0; q < budget; q++) {
                int s = order[q];
                WaveIn wi;
                wi.gtotal = c[s].gtotal;
                wi.begin = c[s].begin; wi.end = c[s].end; wi.feat = c[s].feat; wi.thr = c[s].bin;
                wi.parent_slot = c[s].dslot;
                wi.left_slot = pool.take(); wi.right_slot = pool.take();
                wi.depth_ok = (c[s].depth + 1) < P->max_depth;
                win.push_back(wi);
                who.push_back(s);
            }
            TRY(device_wave(ctx, rf, win, P, nl, kids));
            for (size_t q = 0; q < who.size(); q++) {
                Cand &x = c[who[q]];
                x.expanded = 1;
                x.nl = nl[q];
                x.nr = (x.end - x.begin) - nl[q];
                x.kid[0] = kids[2 * q];
                x.kid[1] = kids[2 * q + 1];
                x.kslot[0] = win[q].left_slot;
                x.kslot[1] = win[q].right_slot;
            }
            if (!c[ci].expanded) return fail(ctx, GBM_ERR_STATE, "internal: selected node not expanded");
        }
        Cand &pc = c[ci];
        int cur = pc.node;
        long long gnl = pc.kid[0].n, gnr = pc.kid[1].n;   // global counts
        if (gnl < msl || gnr < msl) {                      // E:678-683
            T.tf[cur] = -1; T.tv[cur] = pc.val; pc.active = false;
            pool.give(pc.kslot[0]); pool.give(pc.kslot[1]); pool.give(pc.dslot);
            continue;
        }
        int lid = node_count++, rid = node_count++;
        T.tf[cur] = pc.feat; T.tt[cur] = pc.bin; T.tl[cur] = lid; T.tr[cur] = rid;
        T.tv[cur] = pc.val; T.sg[cur] = pc.gain;
        n_splits++;
        ctx->alg_bytes += (double)std::min(gnl, gnr) * (rf.nf + 8);
        int nd = pc.depth + 1;
        bool left_small = gnl <= gnr;
        int ss = -1, sl = -1;                              // E:712-720
        for (int s = 0; s < MAXC; s++) {
            if (s != ci && !c[s].active) {
                if (ss < 0) ss = s; else if (sl < 0) { sl = s; break; }
            }
        }
        Cand parent = pc;
        pool.give(parent.dslot);
        c[ci].active = false;
        for (int pass = 0; pass < 2; pass++) {
            int side = (pass == 0) == left_small ? 0 : 1;   // 0 = left
            int slot = pass == 0 ? ss : sl;
            const ChildRes &k = parent.kid[side];
            Cand &x = c[slot];
            x = Cand();
            x.node = side == 0 ? lid : rid;
            x.depth = nd;
            x.val = -k.G / (k.H + lam);
            bool can = k.n >= msl && k.H >= mcw && nd < P->max_depth;
            x.feat = (can && k.feat >= 0) ? k.feat : -1;
            x.bin = (can && k.feat >= 0) ? k.bin : 0;
            x.gain = (can && k.feat >= 0) ? k.gain : -1.0;
            x.active = true;
            x.dslot = parent.kslot[side];
            long long lbeg = parent.begin, lmid = parent.begin + parent.nl;
            x.begin = side == 0 ? lbeg : lmid;
            x.end = side == 0 ? lmid : parent.end;
            x.gtotal = k.n;
        }
    }
    for (int s = 0; s < MAXC; s++)
        if (c[s].active) { T.tf[c[s].node] = -1; T.tv[c[s].node] = c[s].val; }
    T.nc = node_count;
    return GBM_OK;
}

// Depth-wise DFS builder (E:233-508): every splittable node of a level is
// expanded in one wave; node ids are then assigned in the reference's DFS
// order (smaller child popped first).
struct DNode {
    long long begin, end;
    int depth, dslot;
    ChildRes r;             // totals + best split
    int expanded = 0;
    long long nl = 0;
    int kid[2] = {-1, -1};  // indices into the node list
    int kslot[2] = {-1, -1};
};

int build_depthwise(gbm_ctx *ctx, const RoundFeat &rf, long long n_sub, long long n_sub_g,
                    const gbm_params *P, HostTree &T) {
    const double lam = P->reg_lambda, mcw = P->min_child_weight;
    const long long msl = P->min_samples_leaf;
    const int D = P->max_depth;
    T.init((1 << (D + 1)) - 1);
    SlotPool pool;
    pool.reset(ctx->pool_slots);
    std::vector<DNode> nodes;
    DNode root;
    root.begin = 0; root.end = n_sub; root.depth = 0; root.dslot = pool.take();
    TRY(device_root(ctx, rf, n_sub, n_sub_g, root.dslot, D > 0, P, root.r));
    nodes.push_back(root);
    auto splittable = [&](const DNode &x) {
        return !(x.depth >= D || x.r.n < msl || x.r.H < mcw) && x.r.feat >= 0;
    };
    std::vector<int> level = {0};
    std::vector<long long> nl;
    std::vector<ChildRes> kids;
    while (!level.empty()) {
        std::vector<int> todo;
        for (int id : level) if (splittable(nodes[id])) todo.push_back(id);
        std::vector<int> next;
        for (size_t b0 = 0; b0 < todo.size();) {
            int cnt = (int)std::min<size_t>(todo.size() - b0,
                                            (size_t)std::min(std::min(kMaxWave, ctx->stage_slots),
                                                             pool.avail() / 2));
            if (cnt < 1) return fail(ctx, GBM_ERR_STATE, "histogram slot pool exhausted");
            std::vector<WaveIn> win;
            for (int q = 0; q < cnt; q++) {
                DNode &x = nodes[todo[b0 + q]];
                WaveIn wi;
                wi.gtotal = x.r.n;
                wi.begin = x.begin; wi.end = x.end; wi.feat = x.r.feat; wi.thr = x.r.bin;
                wi.parent_slot = x.dslot; wi.left_slot = pool.take(); wi.right_slot = pool.take();
                wi.depth_ok = (x.depth + 1) < D;
                win.push_back(wi);
            }
            TRY(device_wave(ctx, rf, win, P, nl, kids));
            for (int q = 0; q < cnt; q++) {
                int id = todo[b0 + q];
                pool.give(nodes[id].dslot);
                nodes[id].expanded = 1;
                nodes[id].nl = nl[q];
                long long gl = kids[2 * q].n, gr = kids[2 * q + 1].n;
                if (gl < msl || gr < msl) {     // E:439-443: becomes a leaf
                    pool.give(win[q].left_slot); pool.give(win[q].right_slot);
                    nodes[id].expanded = 2;
                    continue;
                }
                for (int s = 0; s < 2; s++) {
                    DNode ch;
                    ch.begin = s == 0 ? nodes[id].begin : nodes[id].begin + nl[q];
                    ch.end = s == 0 ? nodes[id].begin + nl[q] : nodes[id].end;
                    ch.depth = nodes[id].depth + 1;
                    ch.dslot = s == 0 ? win[q].left_slot : win[q].right_slot;
                    ch.r = kids[2 * q + s];
                    nodes[id].kid[s] = (int)nodes.size();
                    nodes.push_back(ch);
                    next.push_back(nodes[id].kid[s]);
                }
            }
            b0 += cnt;
        }
        // children that will not split release their histograms now
        for (int id : next) if (!splittable(nodes[id])) { pool.give(nodes[id].dslot); nodes[id].dslot = -1; }
        level.swap(next);
    }
    // DFS numbering exactly as the reference's stack (E:287-505)
    int node_count = 0;
    struct SE { int id, tid; };
    std::vector<SE> stack;
    stack.push_back({0, node_count++});
    while (!stack.empty()) {
        SE e = stack.back();
        stack.pop_back();
        DNode &x = nodes[e.id];
        double val = -x.r.G / (x.r.H + lam);
        if (x.expanded != 1) { T.tf[e.tid] = -1; T.tv[e.tid] = val; continue; }
        int lid = node_count++, rid = node_count++;
        ctx->alg_bytes += (double)std::min(nodes[x.kid[0]].r.n, nodes[x.kid[1]].r.n) * (rf.nf + 8);
        T.tf[e.tid] = x.r.feat; T.tt[e.tid] = x.r.bin; T.tl[e.tid] = lid; T.tr[e.tid] = rid;
        T.tv[e.tid] = val; T.sg[e.tid] = x.r.gain;
        long long gl = nodes[x.kid[0]].r.n, gr = nodes[x.kid[1]].r.n;
        bool left_small = gl <= gr;
        int small = left_small ? 0 : 1;
        stack.push_back({x.kid[1 - small], small == 0 ? rid : lid});   // larger pushed first
        stack.push_back({x.kid[small], small == 0 ? lid : rid});       // smaller popped first
    }
    T.nc = node_count;
    return GBM_OK;
}

void post_prune(HostTree &T, double gamma) {     // E:827-841
    for (int k = T.nc - 1; k >= 0; k--) {
        if (T.tf[k] != -1) {
            int l = T.tl[k], r = T.tr[k];
            if (T.tf[l] == -1 && T.tf[r] == -1 && T.sg[k] < gamma) { T.tf[k] = -1; T.tl[k] = -1; T.tr[k] = -1; }
        }
    }
}

void enforce_monotone(HostTree &T, const int32_t *mono) {   // E:2461-2499
    if (!mono) return;
    for (int k = 0; k < T.nc; k++) {
        int f = T.tf[k];
        if (f < 0) continue;
        int c = mono[f];
        if (c == 0) continue;
        int l = T.tl[k], r = T.tr[k];
        if (l < 0 || r < 0) continue;
        double lv = T.tv[l], rv = T.tv[r];
        if (c == 1) {
            if (lv > rv) { double m = (lv + rv) / 2.0; T.tv[l] = m; T.tv[r] = m; }
        } else if (c == -1 && lv < rv) {
            double m = (lv + rv) / 2.0; T.tv[l] = m; T.tv[r] = m;
        }
    }
}

int alloc_round_fixed(gbm_ctx *ctx) {
    TRY(dalloc(ctx, &ctx->d_mask, (size_t)ctx->n));
    TRY(dalloc(ctx, &ctx->d_rows, (size_t)ctx->n));
    TRY(dalloc(ctx, &ctx->d_tmp, (size_t)ctx->n));
    int ntile = (int)((ctx->n + kCompTile - 1) / kCompTile);
    TRY(dalloc(ctx, &ctx->d_cnt, (size_t)ntile));
    TRY(dalloc(ctx, &ctx->d_off, (size_t)ntile));
    TRY(dalloc(ctx, &ctx->d_total, 1));
    TRY(dalloc(ctx, &ctx->d_blist, (size_t)ctx->nblk));
    TRY(dalloc(ctx, &ctx->d_fpos, (size_t)ctx->nblk * kBlk));
    TRY(dalloc(ctx, &ctx->d_htask, (size_t)kMaxWave));
    TRY(dalloc(ctx, &ctx->d_hprefix, (size_t)kMaxWave + 1));
    TRY(dalloc(ctx, &ctx->d_ptask, (size_t)kMaxWave));
    TRY(dalloc(ctx, &ctx->d_nleft, (size_t)kMaxWave));
    TRY(dalloc(ctx, &ctx->d_nleft_g, (size_t)kMaxWave));
    TRY(dalloc(ctx, &ctx->d_gtot, (size_t)kMaxWave));
    TRY(dalloc(ctx, &ctx->d_count, 1));
    TRY(dalloc(ctx, &ctx->d_child_n, (size_t)2 * kMaxWave));
    TRY(dalloc(ctx, &ctx->d_wave, (size_t)kMaxWave));
    TRY(dalloc(ctx, &ctx->d_stask, (size_t)2 * kMaxWave));
    TRY(dalloc(ctx, &ctx->d_sout, (size_t)2 * kMaxWave));
    TRY(dalloc(ctx, &ctx->d_tree, 1));
    TRY(dalloc(ctx, &ctx->d_leaf, (size_t)ctx->n));
    ctx->upd_blocks = grid_for(ctx->n, kUpdThreads, 148 * 8);
    TRY(dalloc(ctx, &ctx->d_loss_part, (size_t)ctx->upd_blocks));
    TRY(dalloc(ctx, &ctx->d_loss, 1));
    TRY(halloc(ctx, &ctx->h_sout, (size_t)2 * kMaxWave));
    TRY(halloc(ctx, &ctx->h_nleft, (size_t)2 * kMaxWave));
    TRY(halloc(ctx, &ctx->h_nloc, (size_t)kMaxWave));
    TRY(halloc(ctx, &ctx->h_count, 1));
    TRY(halloc(ctx, &ctx->h_loss, 1));
    TRY(halloc(ctx, &ctx->h_total, 1));
    TRY(halloc(ctx, &ctx->h_mask, (size_t)ctx->n));
    ctx->tile_cap = 0;
    return GBM_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" {

int gbm_ctx_create(int32_t device, gbm_ctx **out) {
    if (!out) return GBM_ERR_ARG;
    *out = nullptr;
    gbm_ctx *ctx = new (std::nothrow) gbm_ctx();
    if (!ctx) return GBM_ERR_ALLOC;
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev <= 0 || device < 0 || device >= ndev) {
        *out = ctx;   // returned so the caller can read the message
        return fail(ctx, GBM_ERR_CUDA, "CUDA device %d unavailable (%d devices): %s", device, ndev,
                    cudaGetErrorString(e));
    }
    ctx->dev = device;
    *out = ctx;
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&ctx->st, cudaStreamNonBlocking));
    CK(cudaFuncSetAttribute(k_hist, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            kBlk * kBins * 2 * (int)sizeof(unsigned long long)));
    return GBM_OK;
}

const char *gbm_last_error(const gbm_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

void gbm_ctx_destroy(gbm_ctx *ctx) {
    if (!ctx) return;
    if (ctx->dev >= 0) {
        cudaSetDevice(ctx->dev);
        if (ctx->st) cudaStreamSynchronize(ctx->st);
    }
    if (ctx->comm) gbm_comm_destroy(ctx->comm);
    void *dev_ptrs[] = {ctx->d_xb, ctx->d_counts, ctx->d_y, ctx->d_F, ctx->d_q, ctx->d_mask, ctx->d_rows,
                        ctx->d_tmp, ctx->d_cnt, ctx->d_off, ctx->d_total, ctx->d_blist, ctx->d_fidx,
                        ctx->d_fpos, ctx->d_pool, ctx->d_stage, ctx->d_htask, ctx->d_hprefix, ctx->d_ptask,
                        ctx->d_tile_cnt, ctx->d_tile_off, ctx->d_nleft, ctx->d_nleft_g, ctx->d_gtot,
                        ctx->d_count, ctx->d_child_n, ctx->d_wave,
                        ctx->d_stask, ctx->d_sout, ctx->d_tree, ctx->d_leaf, ctx->d_loss_part, ctx->d_loss,
                        ctx->d_px, ctx->d_pnodes, ctx->d_pvals, ctx->d_poff, ctx->d_pF, ctx->d_pP};
    for (void *p : dev_ptrs) if (p) cudaFree(p);
    void *host_ptrs[] = {ctx->h_sout, ctx->h_nleft, ctx->h_nloc, ctx->h_count, ctx->h_loss, ctx->h_total,
                         ctx->h_mask};
    for (void *p : host_ptrs) if (p) cudaFreeHost(p);
    for (cudaEvent_t e : ctx->hist_ev) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->mark) if (e) cudaEventDestroy(e);
    if (ctx->st) cudaStreamDestroy(ctx->st);
    delete ctx;
}

int gbm_sync(gbm_ctx *ctx) {
    if (!ctx || ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    return sync_stream(ctx);
}

int gbm_ctx_init_comm(gbm_ctx *ctx, const void *uid, int32_t nranks, int32_t rank, int32_t timeout_ms) {
    if (!ctx || !uid || nranks < 1 || rank < 0 || rank >= nranks) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    ctx->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
    if (nranks == 1) return GBM_OK;
    return gbm_comm_create(&ctx->comm, uid, nranks, rank, ctx->timeout_ms, ctx->err);
}

int gbm_nccl_unique_id(void *uid_out) { return gbm_comm_unique_id(uid_out); }

int gbm_upload_bins(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p, const int32_t *bin_counts) {
    if (!ctx || !xbin || !bin_counts || n <= 0 || p <= 0 || n > 0x7fffffffLL) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    for (int j = 0; j < p; j++)
        if (bin_counts[j] < 1 || bin_counts[j] > kBins)
            return fail(ctx, GBM_ERR_UNSUPPORTED, "feature %d has %d bins; the device path holds 1..256 bins",
                        j, bin_counts[j]);
    CK(cudaSetDevice(ctx->dev));
    ctx->n = n; ctx->p = p; ctx->nblk = (p + kBlk - 1) / kBlk;
    ctx->counts.assign(bin_counts, bin_counts + p);
    TRY(dalloc(ctx, &ctx->d_xb, (size_t)ctx->nblk * n * kBlk));
    TRY(dalloc(ctx, &ctx->d_counts, (size_t)p));
    CK(cudaMemcpyAsync(ctx->d_counts, bin_counts, sizeof(int32_t) * p, cudaMemcpyHostToDevice, ctx->st));
    // stream row chunks through a staging buffer and transpose to column blocks
    int64_t chunk_rows = std::max<int64_t>(1, (int64_t)(64 << 20) / p);
    chunk_rows = std::min(chunk_rows, n);
    uint8_t *stage = nullptr;
    TRY(dalloc(ctx, &stage, (size_t)(chunk_rows * p)));
    int rc = GBM_OK;
    for (int64_t r0 = 0; r0 < n && rc == GBM_OK; r0 += chunk_rows) {
        int64_t rows = std::min(chunk_rows, n - r0);
        cudaError_t e = cudaMemcpyAsync(stage, xbin + r0 * p, (size_t)(rows * p), cudaMemcpyHostToDevice, ctx->st);
        if (e != cudaSuccess) { rc = fail(ctx, GBM_ERR_CUDA, "bin upload: %s", cudaGetErrorString(e)); break; }
        k_pack_bins<<<grid_for(rows * ctx->nblk, 256), 256, 0, ctx->st>>>(stage, rows, p, r0, n, ctx->nblk,
                                                                           ctx->d_counts, ctx->d_xb);
        e = cudaGetLastError();
        if (e != cudaSuccess) { rc = fail(ctx, GBM_ERR_CUDA, "k_pack_bins: %s", cudaGetErrorString(e)); break; }
        e = cudaStreamSynchronize(ctx->st);
        if (e != cudaSuccess) { rc = fail(ctx, GBM_ERR_CUDA, "bin upload sync: %s", cudaGetErrorString(e)); break; }
    }
    cudaFree(stage);
    if (rc != GBM_OK) return rc;
    TRY(alloc_round_fixed(ctx));
    TRY(dalloc(ctx, &ctx->d_y, (size_t)n));
    TRY(dalloc(ctx, &ctx->d_F, (size_t)n));
    TRY(dalloc(ctx, &ctx->d_q, (size_t)n));
    ctx->have_bins = true;
    ctx->have_labels = false;
    return GBM_OK;
}

int gbm_upload_labels(gbm_ctx *ctx, const uint8_t *y, const double class_w[2], double base_score,
                      int64_t n_global) {
    if (!ctx || !y || !class_w) return GBM_ERR_ARG;
    if (!ctx->have_bins) return fail(ctx, GBM_ERR_STATE, "upload bins before labels");
    if (!(class_w[0] > 0.0) || !(class_w[1] > 0.0) || !std::isfinite(class_w[0]) || !std::isfinite(class_w[1]))
        return fail(ctx, GBM_ERR_ARG, "class weights must be finite and > 0");
    CK(cudaSetDevice(ctx->dev));
    ctx->w[0] = class_w[0]; ctx->w[1] = class_w[1];
    ctx->base = base_score;
    ctx->n_global = n_global > 0 ? n_global : ctx->n;
    ctx->S = scale_bits_for(std::max(class_w[0], class_w[1]));
    CK(cudaMemcpyAsync(ctx->d_y, y, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    std::vector<double> F0((size_t)ctx->n, base_score);
    CK(cudaMemcpyAsync(ctx->d_F, F0.data(), sizeof(double) * ctx->n, cudaMemcpyHostToDevice, ctx->st));
    double scale = std::ldexp(1.0, ctx->S);
    k_init_grad<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_F, ctx->d_y, ctx->n, ctx->w[0], ctx->w[1],
                                                             scale, ctx->d_q);
    CKL();
    TRY(sync_stream(ctx));
    ctx->have_labels = true;
    return GBM_OK;
}

int32_t gbm_scale_bits(const gbm_ctx *ctx) { return ctx ? ctx->S : 0; }

int gbm_get_F(gbm_ctx *ctx, double *F_out) {
    if (!ctx || !F_out) return GBM_ERR_ARG;
    if (!ctx->have_labels) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    CK(cudaMemcpyAsync(F_out, ctx->d_F, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st));
    return sync_stream(ctx);
}

int gbm_get_grad(gbm_ctx *ctx, double *g_out, double *h_out) {
    if (!ctx || !g_out || !h_out) return GBM_ERR_ARG;
    if (!ctx->have_labels) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    double *dg = nullptr, *dh = nullptr;
    TRY(dalloc(ctx, &dg, (size_t)ctx->n));
    int rc = dalloc(ctx, &dh, (size_t)ctx->n);
    if (rc != GBM_OK) { cudaFree(dg); return rc; }
    k_export_grad<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_F, ctx->d_y, ctx->n, ctx->w[0], ctx->w[1], dg, dh);
    cudaMemcpyAsync(g_out, dg, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
    cudaMemcpyAsync(h_out, dh, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
    cudaError_t e = cudaStreamSynchronize(ctx->st);
    cudaFree(dg);
    cudaFree(dh);
    if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "gbm_get_grad: %s", cudaGetErrorString(e));
    return GBM_OK;
}

}  // extern "C"

namespace {

int check_tree_args(gbm_ctx *ctx, int32_t nfeat, const gbm_params *P, const gbm_tree_out *out) {
    if (nfeat <= 0 || nfeat > ctx->p) return fail(ctx, GBM_ERR_ARG, "nfeat=%d out of range", nfeat);
    if (P->max_leaves < 2 && P->grow_policy == 0) return fail(ctx, GBM_ERR_ARG, "max_leaves must be >= 2");
    if (P->max_depth <= 0) return fail(ctx, GBM_ERR_ARG, "max_depth must be > 0");
    if (P->grow_policy == 1 && P->max_depth > 7)
        return fail(ctx, GBM_ERR_UNSUPPORTED, "depth-wise trees deeper than 7 are not supported");
    if (P->grow_policy == 0 && P->max_leaves > 127)
        return fail(ctx, GBM_ERR_UNSUPPORTED, "max_leaves > 127 is not supported");
    int need = P->grow_policy == 0 ? 2 * P->max_leaves + 2 : (1 << (P->max_depth + 1)) - 1;
    if (out->capacity < need) return fail(ctx, GBM_ERR_ARG, "tree capacity %d < %d", out->capacity, need);
    return GBM_OK;
}

// In-bag compaction, tree growth, prune and monotone clipping.  Leaves the
// pruned tree in T.
int grow_tree(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
              const gbm_params *P, HostTree &T) {
    CK(cudaSetDevice(ctx->dev));
    int leaves_for_pool = P->grow_policy == 0 ? P->max_leaves : (1 << std::min(P->max_depth, 7));
    TRY(ensure_round_buffers(ctx, nfeat, leaves_for_pool));
    RoundFeat rf;
    TRY(setup_features(ctx, feat_idx, nfeat, rf));

    // in-bag rows -> sorted row list
    std::memcpy(ctx->h_mask, inbag_mask, (size_t)ctx->n);
    CK(cudaMemcpyAsync(ctx->d_mask, ctx->h_mask, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    int ntile = (int)((ctx->n + kCompTile - 1) / kCompTile);
    k_comp_count<<<ntile, 256, 0, ctx->st>>>(ctx->d_mask, ctx->n, ctx->d_cnt);
    CKL();
    k_scan_small<<<1, 1024, 0, ctx->st>>>(ctx->d_cnt, ntile, ctx->d_off, ctx->d_total);
    CKL();
    k_comp_scatter<<<ntile, 256, 0, ctx->st>>>(ctx->d_mask, ctx->n, ctx->d_off, ctx->d_rows);
    CKL();
    CK(cudaMemcpyAsync(ctx->h_total, ctx->d_total, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    long long n_sub = ctx->h_total[0];
    long long n_sub_g = n_sub;
    if (ctx->comm) {
        TRY(gbm_comm_check_alive(ctx->comm, ctx->timeout_ms, ctx->err));
        ctx->h_count[0] = n_sub;
        CK(cudaMemcpyAsync(ctx->d_count, ctx->h_count, sizeof(long long), cudaMemcpyHostToDevice, ctx->st));
        TRY(gbm_comm_allreduce_i64(ctx->comm, ctx->d_count, 1, ctx->st, ctx->timeout_ms, ctx->err));
        CK(cudaMemcpyAsync(ctx->h_count, ctx->d_count, sizeof(long long), cudaMemcpyDeviceToHost, ctx->st));
        TRY(sync_stream(ctx));
        n_sub_g = ctx->h_count[0];
    }

    if (P->grow_policy == 0) TRY(build_leafwise(ctx, rf, n_sub, n_sub_g, P, T));
    else TRY(build_depthwise(ctx, rf, n_sub, n_sub_g, P, T));
    post_prune(T, P->gamma);
    enforce_monotone(T, P->monotone);
    return GBM_OK;
}

void write_tree(const HostTree &T, int need, gbm_tree_out *out) {
    for (int k = 0; k < need; k++) {
        bool in = k < (int)T.tf.size();
        out->tf[k] = in ? T.tf[k] : -1;
        out->tt[k] = in ? T.tt[k] : 0;
        out->tv[k] = in ? T.tv[k] : 0.0;
        out->tl[k] = in ? T.tl[k] : -1;
        out->tr[k] = in ? T.tr[k] : -1;
        out->sg[k] = in ? T.sg[k] : 0.0;
    }
    out->n_nodes = T.nc;
}

int tree_need(const gbm_params *P) {
    return P->grow_policy == 0 ? 2 * P->max_leaves + 2 : (1 << (P->max_depth + 1)) - 1;
}

}  // namespace

extern "C" {

int gbm_build_tree(gbm_ctx *ctx, const double *grad, const double *hess, const uint8_t *inbag_mask,
                   const int32_t *feat_idx, int32_t nfeat, const gbm_params *P, gbm_tree_out *out) {
    if (!ctx || !grad || !hess || !inbag_mask || !feat_idx || !P || !out) return GBM_ERR_ARG;
    if (!ctx->have_bins) return fail(ctx, GBM_ERR_STATE, "upload bins before gbm_build_tree");
    TRY(check_tree_args(ctx, nfeat, P, out));
    CK(cudaSetDevice(ctx->dev));
    double m = 1.0;
    for (int64_t i = 0; i < ctx->n; i++) {
        double a = std::fabs(grad[i]), b = std::fabs(hess[i]);
        if (!std::isfinite(a) || !std::isfinite(b))
            return fail(ctx, GBM_ERR_ARG, "grad/hess[%lld] is not finite", (long long)i);
        m = std::max(m, std::max(a, b));
    }
    ctx->S = scale_bits_for(m);
    double *dg = nullptr, *dh = nullptr;
    TRY(dalloc(ctx, &dg, (size_t)ctx->n));
    int rc = dalloc(ctx, &dh, (size_t)ctx->n);
    if (rc == GBM_OK) {
        cudaMemcpyAsync(dg, grad, sizeof(double) * ctx->n, cudaMemcpyHostToDevice, ctx->st);
        cudaMemcpyAsync(dh, hess, sizeof(double) * ctx->n, cudaMemcpyHostToDevice, ctx->st);
        k_quant<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(dg, dh, ctx->n, std::ldexp(1.0, ctx->S), ctx->d_q);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->st);
        if (e != cudaSuccess) rc = fail(ctx, GBM_ERR_CUDA, "gbm_build_tree upload: %s", cudaGetErrorString(e));
    }
    cudaFree(dg);
    cudaFree(dh);
    if (rc != GBM_OK) return rc;
    ctx->have_labels = false;   // the device gradients no longer follow F
    HostTree T;
    TRY(grow_tree(ctx, inbag_mask, feat_idx, nfeat, P, T));
    write_tree(T, tree_need(P), out);
    return GBM_OK;
}

int gbm_round(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
              const gbm_params *P, gbm_tree_out *out, double *train_loss) {
    if (!ctx || !inbag_mask || !feat_idx || !P || !out) return GBM_ERR_ARG;
    if (!ctx->have_labels) return fail(ctx, GBM_ERR_STATE, "upload bins and labels before gbm_round");
    TRY(check_tree_args(ctx, nfeat, P, out));
    HostTree T;
    TRY(grow_tree(ctx, inbag_mask, feat_idx, nfeat, P, T));
    int need = tree_need(P);

    // F update + loss + next gradients
    TreeDev td;
    std::memset(&td, 0, sizeof td);
    if (T.nc > 256) return fail(ctx, GBM_ERR_UNSUPPORTED, "tree with %d nodes exceeds 256", T.nc);
    td.n = T.nc;
    for (int k = 0; k < T.nc; k++) {
        td.feat[k] = T.tf[k];
        td.thr[k] = (int)std::min<int64_t>(T.tt[k], 255);
        td.left[k] = T.tl[k];
        td.right[k] = T.tr[k];
        td.val[k] = T.tv[k];
    }
    CK(cudaMemcpyAsync(ctx->d_tree, &td, sizeof td, cudaMemcpyHostToDevice, ctx->st));
    double scale = std::ldexp(1.0, ctx->S);
    k_update<<<ctx->upd_blocks, kUpdThreads, 0, ctx->st>>>(
        ctx->d_tree, ctx->d_xb, ctx->n, ctx->d_y, ctx->w[0], ctx->w[1], P->learning_rate, scale, ctx->d_F,
        ctx->d_q, out->leaf_of_row ? ctx->d_leaf : nullptr, ctx->d_loss_part);
    CKL();
    k_sum_partials<<<1, 256, 0, ctx->st>>>(ctx->d_loss_part, ctx->upd_blocks, ctx->d_loss);
    CKL();
    if (ctx->comm) TRY(gbm_comm_allreduce_f64(ctx->comm, ctx->d_loss, 1, ctx->st, ctx->timeout_ms, ctx->err));
    CK(cudaMemcpyAsync(ctx->h_loss, ctx->d_loss, sizeof(double), cudaMemcpyDeviceToHost, ctx->st));
    if (out->leaf_of_row)
        CK(cudaMemcpyAsync(out->leaf_of_row, ctx->d_leaf, sizeof(int32_t) * ctx->n, cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    if (train_loss) *train_loss = -ctx->h_loss[0] / (double)ctx->n_global;
    write_tree(T, need, out);
    return GBM_OK;
}

// ---- predict ------------------------------------------------------------------

int gbm_predict_set_model(gbm_ctx *ctx, const gbm_packed *m, int32_t n_features) {
    if (!ctx || !m || m->n_trees < 0 || !m->offsets) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    int32_t T = m->n_trees;
    int64_t total = m->offsets[T];
    std::vector<PNode> nodes((size_t)std::max<int64_t>(total, 1));
    std::vector<double> vals((size_t)std::max<int64_t>(total, 1));
    for (int32_t t = 0; t < T; t++) {
        int32_t o = m->offsets[t], o1 = m->offsets[t + 1];
        if (o1 - o > 32767 || o1 < o) return fail(ctx, GBM_ERR_UNSUPPORTED, "tree %d has %d nodes", t, o1 - o);
        for (int32_t k = o; k < o1; k++) {
            PNode nd;
            nd.feat = m->features[k];
            int64_t th = m->thresholds[k];
            nd.thr = (uint8_t)(th < 0 ? 0 : (th > 255 ? 255 : th));
            nd.pad = 0;
            nd.left = (int16_t)m->left[k];
            nd.right = (int16_t)m->right[k];
            if (nd.feat >= 0) {
                if (nd.feat >= n_features) return fail(ctx, GBM_ERR_ARG, "node feature %d >= %d", nd.feat, n_features);
                if (th < 0) return fail(ctx, GBM_ERR_UNSUPPORTED, "negative threshold");
                if (m->left[k] < 0 || m->left[k] >= o1 - o || m->right[k] < 0 || m->right[k] >= o1 - o)
                    return fail(ctx, GBM_ERR_ARG, "tree %d node %d has an out-of-range child", t, k - o);
            }
            nodes[(size_t)k] = nd;
            vals[(size_t)k] = m->values[k];
        }
    }
    if (total > ctx->p_nodes_cap) {
        TRY(dalloc(ctx, &ctx->d_pnodes, (size_t)total));
        TRY(dalloc(ctx, &ctx->d_pvals, (size_t)total));
        ctx->p_nodes_cap = total;
    }
    if (T + 1 > ctx->p_trees_cap) {
        TRY(dalloc(ctx, &ctx->d_poff, (size_t)T + 1));
        ctx->p_trees_cap = T + 1;
    }
    CK(cudaMemcpyAsync(ctx->d_pnodes, nodes.data(), sizeof(PNode) * total, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_pvals, vals.data(), sizeof(double) * total, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_poff, m->offsets, sizeof(int32_t) * (T + 1), cudaMemcpyHostToDevice, ctx->st));
    ctx->p_ntree = T;
    ctx->p_nfeat = n_features;
    return sync_stream(ctx);
}

int gbm_predict_upload(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p) {
    if (!ctx || !xbin || n <= 0 || p <= 0) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    if (ctx->p_nfeat && p != ctx->p_nfeat) return fail(ctx, GBM_ERR_ARG, "X has %d features, model %d", p, ctx->p_nfeat);
    CK(cudaSetDevice(ctx->dev));
    if (n * p > ctx->pn_cap) {
        TRY(dalloc(ctx, &ctx->d_px, (size_t)(n * p)));
        ctx->pn_cap = n * p;
    }
    TRY(dalloc(ctx, &ctx->d_pF, (size_t)n));
    TRY(dalloc(ctx, &ctx->d_pP, (size_t)n));
    CK(cudaMemcpyAsync(ctx->d_px, xbin, (size_t)(n * p), cudaMemcpyHostToDevice, ctx->st));
    ctx->pn = n;
    ctx->pp = p;
    return GBM_OK;
}

int gbm_predict_run(gbm_ctx *ctx, double lr, double base) {
    if (!ctx) return GBM_ERR_ARG;
    if (!ctx->d_px || !ctx->d_poff) return fail(ctx, GBM_ERR_STATE, "upload a model and rows first");
    CK(cudaSetDevice(ctx->dev));
    k_predict<<<grid_for(ctx->pn, 256), 256, 0, ctx->st>>>(ctx->d_px, ctx->pn, ctx->pp, ctx->d_pnodes, ctx->d_pvals,
                                                          ctx->d_poff, ctx->p_ntree, lr, base, ctx->d_pF, ctx->d_pP);
    CKL();
    return GBM_OK;
}

int gbm_predict_fetch(gbm_ctx *ctx, double *F_out, double *proba_out) {
    if (!ctx) return GBM_ERR_ARG;
    CK(cudaSetDevice(ctx->dev));
    if (F_out) CK(cudaMemcpyAsync(F_out, ctx->d_pF, sizeof(double) * ctx->pn, cudaMemcpyDeviceToHost, ctx->st));
    if (proba_out) CK(cudaMemcpyAsync(proba_out, ctx->d_pP, sizeof(double) * ctx->pn, cudaMemcpyDeviceToHost, ctx->st));
    return sync_stream(ctx);
}

int gbm_predict(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p, const gbm_packed *model, double lr,
                double base, double *F_out, double *proba_out) {
    TRY(gbm_predict_set_model(ctx, model, p));
    TRY(gbm_predict_upload(ctx, xbin, n, p));
    TRY(gbm_predict_run(ctx, lr, base));
    return gbm_predict_fetch(ctx, F_out, proba_out);
}

// ---- instrumentation ------------------------------------------------------

int gbm_set_profiling(gbm_ctx *ctx, int32_t on) {
    if (!ctx) return GBM_ERR_ARG;
    ctx->profiling = on != 0;
    return GBM_OK;
}

int gbm_get_stats(gbm_ctx *ctx, gbm_stats *out) {
    if (!ctx || !out) return GBM_ERR_ARG;
    out->kernel_launches = ctx->launches;
    out->hist_launches = ctx->hist_launches;
    out->hist_rows = ctx->hist_rows;
    out->waves = ctx->waves;
    out->hist_ms = ctx->hist_ms;
    out->hist_alg_bytes = ctx->alg_bytes;
    return GBM_OK;
}

int gbm_reset_stats(gbm_ctx *ctx) {
    if (!ctx) return GBM_ERR_ARG;
    ctx->launches = ctx->hist_launches = ctx->hist_rows = ctx->waves = 0;
    ctx->hist_ms = ctx->alg_bytes = 0.0;
    return GBM_OK;
}

int gbm_event_record(gbm_ctx *ctx, int32_t slot) {
    if (!ctx || slot < 0 || slot >= 16) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    if (!ctx->mark[slot]) CK(cudaEventCreate(&ctx->mark[slot]));
    CK(cudaEventRecord(ctx->mark[slot], ctx->st));
    return GBM_OK;
}

int gbm_event_elapsed(gbm_ctx *ctx, int32_t a, int32_t b, float *ms) {
    if (!ctx || !ms || a < 0 || a >= 16 || b < 0 || b >= 16) return GBM_ERR_ARG;
    if (!ctx->mark[a] || !ctx->mark[b]) return fail(ctx, GBM_ERR_STATE, "event slot not recorded");
    CK(cudaSetDevice(ctx->dev));
    CK(cudaEventSynchronize(ctx->mark[b]));
    CK(cudaEventElapsedTime(ms, ctx->mark[a], ctx->mark[b]));
    return GBM_OK;
}

}  // extern "C"
