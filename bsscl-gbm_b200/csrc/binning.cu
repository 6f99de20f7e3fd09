// binning.cu -- bin edges and bin ids on the GPU (binning_internal.h).
//
// Edges follow HybridHistGBMNumbaV1_0_1._build_bin_edges
// (src/bsscl_gbm/estimator_v1_0_1.py, "E" below, E:2073-2141) for
// sample_weight=None:
//   * a feature with NaN reserves bin 0 for it (E:2094-2097); an all-NaN
//     feature gets edges [0, 1] and one bin (E:2098-2103);
//   * with at most max_numeric_bins = n_bins - has_nan distinct values the
//     edges are the sorted distinct values (E:2108-2109), otherwise
//     np.unique(np.percentile(col, linspace(0, 1, max_numeric_bins+1)*100))
//     (E:2111-2126);
//   * the edge e[-1] + 1e-8 is appended in the dtype of e (E:2127): float32
//     for distinct float32 values (a float32 add of float32(1e-8)), float64
//     for percentiles, which NumPy returns as float64;
//   * every row is padded with its last edge (E:2135-2139).
//
// NumPy's percentile ('linear' method, numpy.lib._function_base_impl,
// NumPy 2.3) is restated operation by operation, x being the sorted
// non-NaN values (order statistics: any sort gives the same values):
//   q    = (linspace(0, 1, k) * 100) / 100                      float64
//   v    = (nc - 1) * q                                          float64
//   v >= nc - 1:  a = b = x[nc-1], t = v + 1   (previous index -1)
//   otherwise:    a = x[floor v], b = x[floor v + 1], t = v - floor v
//   d    = b - a                                  in the data's dtype
//   r    = a + d*t;  where t >= 0.5:  r = b - d*(1 - t)          float64
// np.unique then sorts the k results and drops repeats (NaNs collapse into
// one NaN, last).
//
// The sort: every column as order-preserving unsigned keys (sign-magnitude
// mapped to unsigned order; NaN -> all ones, which sorts last) and one radix
// sort per column (CUB).  Distinct values are counted on the keys, -0.0 and
// +0.0 being one value (they compare equal, as in np.unique).
//
// Bin ids follow _bin_features (E:2144-2189) with the 'standard' search of
// bin_all_features_standard_numba (E:204-226): v < e[0] -> 0,
// v >= e[nb] -> nb - 1, else the largest k < nb with e[k] <= v.  The
// 'hybrid' search (E:155-202) accepts its guess only under the same
// condition and so returns the same id.  When any feature had NaN in
// training, NaN is searched as 0.0 and the features with a NaN bin then map
// NaN -> 0 and shift the other ids up by one (E:2157-2172); otherwise NaN
// falls to id 0 of the search.  On the device the search is a branch-free
// binary search over a power-of-two table of e[1..nb-1] padded with NaN
// (never <= v, like the NaN edges np.percentile gives a column holding
// infinities, which np.unique puts last).
// For float32 data the table holds every edge rounded up to float32, which
// decides each comparison with a float32 value exactly as the float64 edge
// does: e <= v  <=>  round_up_f32(e) <= v, and v < e  <=>  v < round_up_f32(e).
#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <vector>

#include "binning_internal.h"
#include "gbm_common.cuh"

namespace gbmbin {

namespace {

constexpr int kMaxBins = 1023;     // n_bins accepted by edges() (k <= 1024 quantiles per feature)
constexpr int kMaxTab = 1024;      // bins per feature accepted by the binning kernels
constexpr int kScanThreads = 512;
constexpr int kScanItems = 4;
constexpr int kFinalThreads = 1024;
constexpr int kBinThreads = 256;

template <typename T>
struct Keys;
template <>
struct Keys<float> {
    typedef uint32_t K;
    typedef float V;   // type of the binning table
    static constexpr K kNaN = 0xffffffffu, kNeg0 = 0x7fffffffu, kPos0 = 0x80000000u;
    static constexpr int kBits = 32;
};
template <>
struct Keys<double> {
    typedef unsigned long long K;
    typedef double V;
    static constexpr K kNaN = 0xffffffffffffffffull, kNeg0 = 0x7fffffffffffffffull, kPos0 = 0x8000000000000000ull;
    static constexpr int kBits = 64;
};

__device__ __forceinline__ uint32_t okey(float v) {
    const uint32_t b = __float_as_uint(v);
    if (v != v) return 0xffffffffu;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ unsigned long long okey(double v) {
    const unsigned long long b = (unsigned long long)__double_as_longlong(v);
    if (v != v) return 0xffffffffffffffffull;
    return (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
}
// inverse of okey (the NaN key decodes to a NaN)
__device__ __forceinline__ float ovalue(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ double ovalue(unsigned long long k) {
    return __longlong_as_double(
        (long long)((k & 0x8000000000000000ull) ? (k & 0x7fffffffffffffffull) : ~k));
}

__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }

// e[-1] + 1e-8 in the dtype of the distinct values (E:2127)
__device__ __forceinline__ double add_eps(double x, float) {
    return (double)__fadd_rn((float)x, static_cast<float>(1e-8));
}
__device__ __forceinline__ double add_eps(double x, double) { return __dadd_rn(x, 1e-8); }

__device__ __forceinline__ float to_tab(double e, float) { return __double2float_ru(e); }
__device__ __forceinline__ double to_tab(double e, double) { return e; }

// NaN-aware order of np.unique: NaN after everything, all NaNs equal
__device__ __forceinline__ bool lt_nan(double a, double b) { return a < b || (a == a && b != b); }
__device__ __forceinline__ bool eq_nan(double a, double b) { return a == b || (a != a && b != b); }

// ---------------------------------------------------------------------------
// edges
// ---------------------------------------------------------------------------

// A row-major chunk [rows][p] -> column-major keys [p][n] at rows r0.. .
template <typename T>
__global__ void __launch_bounds__(256) k_keys(const T *__restrict__ X, int64_t rows, int p, int64_t r0, int64_t n,
                                              typename Keys<T>::K *__restrict__ keys) {
    typedef typename Keys<T>::K K;
    __shared__ K tile[32][33];
    const int64_t i0 = (int64_t)blockIdx.x * 32;
    const int j0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int yy = ty; yy < 32; yy += 8) {
        const int64_t i = i0 + yy;
        const int j = j0 + tx;
        if (i < rows && j < p) tile[yy][tx] = okey(X[i * p + j]);
    }
    __syncthreads();
    for (int yy = ty; yy < 32; yy += 8) {
        const int j = j0 + yy;
        const int64_t i = i0 + tx;
        if (i < rows && j < p) keys[(int64_t)j * n + r0 + i] = tile[tx][yy];
    }
}

// Per feature (one CTA): the non-NaN count and the first `cap` distinct
// values of the sorted column; stops counting once more than n_bins are seen.
template <typename T>
__global__ void __launch_bounds__(kScanThreads) k_edge_scan(const typename Keys<T>::K *__restrict__ sorted, int64_t n,
                                                            const uint8_t *__restrict__ skip, int n_bins, int cap,
                                                            long long *__restrict__ nclean, int *__restrict__ nuniq,
                                                            double *__restrict__ uq) {
    typedef Keys<T> KT;
    typedef typename KT::K K;
    const int j = blockIdx.x;
    if (skip[j]) return;
    const K *col = sorted + (int64_t)j * n;
    __shared__ long long s_nc;
    __shared__ int s_w[32];
    if (threadIdx.x == 0) {   // NaN keys sort last
        int64_t lo = 0, hi = n;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (col[mid] == KT::kNaN) hi = mid;
            else lo = mid + 1;
        }
        s_nc = lo;
    }
    __syncthreads();
    const int64_t nc = s_nc;
    int total = 0;   // distinct values so far (the same in every thread)
    for (int64_t base = 0; base < nc && total <= n_bins; base += (int64_t)kScanItems * kScanThreads) {
        const int64_t i0 = base + (int64_t)threadIdx.x * kScanItems;
        K v[kScanItems];
        K prev = (i0 > 0 && i0 <= nc) ? col[i0 - 1] : (K)0;
        int flags = 0, cnt = 0;
#pragma unroll
        for (int t = 0; t < kScanItems; t++) {
            const int64_t i = i0 + t;
            v[t] = i < nc ? col[i] : (K)0;
            const bool same = prev == v[t] || (prev == KT::kNeg0 && v[t] == KT::kPos0);
            const bool fresh = i < nc && (i == 0 || !same);
            flags |= (int)fresh << t;
            cnt += fresh;
            prev = v[t];
        }
        int tot;
        int off = gbm::block_excl_scan(cnt, s_w, tot);
#pragma unroll
        for (int t = 0; t < kScanItems; t++) {
            if (flags >> t & 1) {
                const int u = total + off++;
                if (u < cap) uq[(int64_t)j * cap + u] = (double)ovalue(v[t]);
            }
        }
        total += tot;
    }
    if (threadIdx.x == 0) {
        nclean[j] = nc;
        nuniq[j] = min(total, cap);
    }
}

// np.percentile of the sorted non-NaN values at one quantile (see the header)
template <typename T>
__device__ double percentile_at(const typename Keys<T>::K *col, int64_t nc, double q) {
    const double nm1 = (double)(nc - 1);
    const double v = __dmul_rn(nm1, q);
    int64_t ia, ib;
    double t;
    if (v >= nm1) {
        ia = ib = nc - 1;
        t = __dadd_rn(v, 1.0);
    } else if (v < 0.0) {
        ia = ib = 0;
        t = v;
    } else {
        const double f = floor(v);
        ia = (int64_t)f;
        ib = ia + 1;
        t = __dsub_rn(v, f);
    }
    const T a = ovalue(col[ia]), b = ovalue(col[ib]);
    const double d = (double)sub_rn(b, a);
    double r = __dadd_rn((double)a, __dmul_rn(d, t));
    if (t >= 0.5) r = __dsub_rn((double)b, __dmul_rn(d, __dsub_rn(1.0, t)));
    return r;
}

// Per feature (one CTA): its edges row, bin count and NaN bin.
template <typename T>
__global__ void __launch_bounds__(kFinalThreads) k_edge_final(const typename Keys<T>::K *__restrict__ sorted, int64_t n,
                                                              const uint8_t *__restrict__ skip, int n_bins, int cap,
                                                              const long long *__restrict__ nclean,
                                                              const int *__restrict__ nuniq,
                                                              const double *__restrict__ uq,
                                                              const double *__restrict__ q_all,
                                                              const double *__restrict__ q_nan,
                                                              double *__restrict__ edges, int stride,
                                                              int *__restrict__ counts, int *__restrict__ nanb) {
    const int j = blockIdx.x;
    if (skip[j]) return;
    __shared__ double r[kFinalThreads];
    __shared__ double e[kFinalThreads + 2];
    __shared__ int keep[kFinalThreads];
    const int tid = threadIdx.x;
    const int64_t nc = nclean[j];
    const bool has_nan = nc < n;
    int len;
    if (nc == 0) {                                   // all NaN (E:2098-2103)
        if (tid == 0) {
            e[0] = 0.0;
            e[1] = 1.0;
        }
        len = 2;
    } else {
        const int mnb = n_bins - (has_nan ? 1 : 0);
        const int nu = nuniq[j];
        if (nu <= mnb) {                             // the distinct values (E:2108-2109)
            for (int u = tid; u < nu; u += blockDim.x) e[u] = uq[(int64_t)j * cap + u];
            if (tid == 0) e[nu] = add_eps(uq[(int64_t)j * cap + nu - 1], T(0));
            len = nu + 1;
        } else {                                     // percentiles (E:2111-2126)
            const int k = mnb + 1;
            const double *q = has_nan ? q_nan : q_all;
            const typename Keys<T>::K *col = sorted + (int64_t)j * n;
            if (tid < k) r[tid] = percentile_at<T>(col, nc, q[tid]);
            __syncthreads();
            bool first = false;
            if (tid < k) {
                first = true;
                for (int t = 0; t < tid; t++)
                    if (eq_nan(r[t], r[tid])) first = false;
                keep[tid] = first;
            }
            __syncthreads();
            if (first) {
                int pos = 0;
                for (int t = 0; t < k; t++) pos += keep[t] && lt_nan(r[t], r[tid]);
                e[pos] = r[tid];
            }
            const int m = __syncthreads_count(first);
            if (tid == 0) e[m] = __dadd_rn(e[m - 1], 1e-8);
            len = m + 1;
        }
    }
    __syncthreads();
    for (int t = tid; t < stride; t += blockDim.x) edges[(int64_t)j * stride + t] = e[min(t, len - 1)];
    if (tid == 0) {
        counts[j] = nc == 0 ? 1 : (has_nan ? len : len - 1);
        nanb[j] = has_nan ? 0 : -1;
    }
}

// ---------------------------------------------------------------------------
// bin ids
// ---------------------------------------------------------------------------

// The search tables of the 16 features of column block `b` in shared memory.
template <typename V>
struct Tab {
    V *tab;   // [16][ts]: e[1..nb-1] as table values, then NaN
    V lo[16], hi[16];
    int nb[16], nanbin[16];
};

template <typename V>
__device__ void build_tab(Tab<V> &T, int b, int p, const double *__restrict__ edges, int stride,
                          const int *__restrict__ counts, const int *__restrict__ nanb, int ts) {
    for (int idx = threadIdx.x; idx < 16 * ts; idx += blockDim.x) {
        const int f = idx / ts, k = idx - f * ts, j = b * 16 + f;
        V val = (V)NAN;
        if (j < p && k < counts[j] - 1) val = to_tab(edges[(int64_t)j * stride + k + 1], V(0));
        T.tab[idx] = val;
    }
    if (threadIdx.x < 16) {
        const int f = threadIdx.x, j = b * 16 + f;
        if (j < p) {
            const int nb = counts[j];
            T.lo[f] = to_tab(edges[(int64_t)j * stride], V(0));
            T.hi[f] = to_tab(edges[(int64_t)j * stride + nb], V(0));
            T.nb[f] = nb;
            T.nanbin[f] = nanb[j] >= 0;
        } else {
            T.lo[f] = T.hi[f] = (V)0;
            T.nb[f] = 1;
            T.nanbin[f] = 0;
        }
    }
    __syncthreads();
}

template <typename V>
__device__ __forceinline__ int search(const V *__restrict__ t, int ts, V lo, V hi, int nb, V x) {
    if (x < lo) return 0;
    if (x >= hi) return nb - 1;
    int pos = 0;
    for (int s = ts >> 1; s > 0; s >>= 1)
        if (t[pos + s - 1] <= x) pos += s;
    return min(pos, nb - 1);
}

// The reference's raw id of value v of feature f of the block.
template <typename V>
__device__ __forceinline__ int bin_id(const Tab<V> &T, int f, int ts, int any_nan, V v) {
    const bool isn = v != v;
    if (any_nan) {
        const int id = search(T.tab + f * ts, ts, T.lo[f], T.hi[f], T.nb[f], isn ? (V)0 : v);
        if (T.nanbin[f]) return isn ? 0 : id + 1;
        return id;
    }
    return search(T.tab + f * ts, ts, T.lo[f], T.hi[f], T.nb[f], v);
}

// Column-major keys rows [lo, lo + rows) -> column blocks uint8 [nblk][rows][16],
// ids clamped to bin_count - 1.
template <typename T>
__global__ void __launch_bounds__(kBinThreads) k_bin_keys(const typename Keys<T>::K *__restrict__ keys, int64_t n,
                                                          int p, int64_t lo, int64_t rows,
                                                          const double *__restrict__ edges, int stride,
                                                          const int *__restrict__ counts,
                                                          const int *__restrict__ nanb, int any_nan, int ts,
                                                          uint8_t *__restrict__ xb, const int32_t *__restrict__ bigidx,
                                                          uint32_t *__restrict__ topbits) {
    typedef typename Keys<T>::V V;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Tab<V> tb;
    if (threadIdx.x == 0) tb.tab = reinterpret_cast<V *>(smem);
    __syncthreads();
    const int b = blockIdx.y;
    build_tab(tb, b, p, edges, stride, counts, nanb, ts);
    const int nf = min(16, p - b * 16);
    for (int64_t i = (int64_t)blockIdx.x * kBinThreads + threadIdx.x; i < rows;
         i += (int64_t)gridDim.x * kBinThreads) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int f = 0; f < nf; f++) {
            const V v = (V)ovalue(keys[(int64_t)(b * 16 + f) * n + lo + i]);
            int id = min(bin_id(tb, f, ts, any_nan, v), tb.nb[f] - 1);
            if (id > 255) {   // bin 256 of a 257-bin feature: stored as 255, marked in the top bits
                atomicOr(topbits + (int64_t)bigidx[b * 16 + f] * ((rows + 31) >> 5) + (i >> 5), 1u << (i & 31));
                id = 255;
            }
            w[f >> 2] |= (uint32_t)id << (8 * (f & 3));
        }
        *reinterpret_cast<uint4 *>(xb + ((int64_t)b * rows + i) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// A row-major chunk [rows][p] -> row-major ids: MODE 0 uint8 clamped to
// bin_count - 1, MODE 1 the raw uint16 ids.
template <typename T, int MODE>
__global__ void __launch_bounds__(kBinThreads) k_bin_rows(const T *__restrict__ X, int64_t rows, int p,
                                                          const double *__restrict__ edges, int stride,
                                                          const int *__restrict__ counts,
                                                          const int *__restrict__ nanb, int any_nan, int ts,
                                                          void *__restrict__ out, const int32_t *__restrict__ bigidx,
                                                          uint32_t *__restrict__ topbits, int64_t row0,
                                                          int64_t top_words) {
    typedef typename Keys<T>::V V;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Tab<V> tb;
    if (threadIdx.x == 0) tb.tab = reinterpret_cast<V *>(smem);
    __syncthreads();
    const int b = blockIdx.y;
    build_tab(tb, b, p, edges, stride, counts, nanb, ts);
    const int nf = min(16, p - b * 16);
    for (int64_t i = (int64_t)blockIdx.x * kBinThreads + threadIdx.x; i < rows;
         i += (int64_t)gridDim.x * kBinThreads) {
        const T *x = X + i * p + b * 16;
        for (int f = 0; f < nf; f++) {
            const int id = bin_id(tb, f, ts, any_nan, (V)x[f]);
            if (MODE == 0) {
                int c = min(id, tb.nb[f] - 1);
                if (c > 255) {   // bin 256 of a 257-bin feature: 255, marked in the top bits
                    const int64_t r = row0 + i;
                    atomicOr(topbits + (int64_t)bigidx[b * 16 + f] * top_words + (r >> 5), 1u << (r & 31));
                    c = 255;
                }
                static_cast<uint8_t *>(out)[i * p + b * 16 + f] = (uint8_t)c;
            }
            else
                static_cast<uint16_t *>(out)[i * p + b * 16 + f] = (uint16_t)id;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int cuda_fail(std::string &err, const char *what, cudaError_t e) {
    err = std::string(what) + ": " + cudaGetErrorString(e);
    return -1;
}

#define BCK(what, call)                                  \
    do {                                                 \
        cudaError_t e_ = (call);                         \
        if (e_ != cudaSuccess) return cuda_fail(err, what, e_); \
    } while (0)

int ensure(void **ptr, size_t &cap, size_t bytes, std::string &err) {
    if (bytes <= cap && *ptr) return 0;
    if (*ptr) cudaFree(*ptr);
    *ptr = nullptr;
    cap = 0;
    cudaError_t e = cudaMalloc(ptr, std::max<size_t>(bytes, 16));
    if (e != cudaSuccess) return cuda_fail(err, "binning buffers", e);
    cap = bytes;
    return 0;
}

// linspace(0, 1, num) * 100 / 100, as NumPy computes it
void quantiles(int num, std::vector<double> &q) {
    q.assign((size_t)num, 0.0);
    const double step = 1.0 / (double)(num - 1);
    for (int i = 0; i < num; i++) {
        double y = (i == num - 1) ? 1.0 : (double)i * step;
        q[(size_t)i] = (y * 100.0) / 100.0;
    }
}

int next_pow2(int x) {
    int t = 1;
    while (t < x) t <<= 1;
    return t;
}

}  // namespace

struct Work {
    int64_t n = 0;
    int p = 0, dtype = -1;
    void *keys = nullptr, *sorted = nullptr, *tmp = nullptr, *stage = nullptr, *ostage = nullptr;
    size_t keys_cap = 0, sorted_cap = 0, tmp_cap = 0, stage_cap = 0, ostage_cap = 0;
    void *small = nullptr;   // per-feature arrays and tables
    size_t small_cap = 0;
};

Work *work_create() { return new Work(); }

void work_destroy(Work *w) {
    if (!w) return;
    for (void *ptr : {w->keys, w->sorted, w->tmp, w->stage, w->ostage, w->small})
        if (ptr) cudaFree(ptr);
    delete w;
}

bool shape(const Work *w, int64_t &n, int &p) {
    if (w->dtype < 0) return false;
    n = w->n;
    p = w->p;
    return true;
}

void release(Work *w) {
    for (void **ptr : {&w->keys, &w->sorted, &w->tmp}) {
        if (*ptr) cudaFree(*ptr);
        *ptr = nullptr;
    }
    w->keys_cap = w->sorted_cap = w->tmp_cap = 0;
    w->dtype = -1;
}

int load(Work *w, gbmh2d::Stager *sg, cudaStream_t st, const void *X, int64_t n, int p, int dtype,
         std::string &err) {
    if (!X || n <= 0 || p <= 0 || n > 0x7fffffffLL || (dtype != 0 && dtype != 1)) {
        err = "binning: bad matrix arguments";
        return -1;
    }
    const size_t ts = dtype ? 8 : 4;
    if (ensure(&w->keys, w->keys_cap, (size_t)n * p * ts, err)) return -1;
    const size_t row = (size_t)p * ts;
    if (row > gbmh2d::chunk_bytes()) {
        err = "binning: rows wider than the upload buffers";
        return -1;
    }
    if (ensure(&w->stage, w->stage_cap, gbmh2d::chunk_bytes(), err)) return -1;
    w->n = n;
    w->p = p;
    w->dtype = dtype;
    void *stage = w->stage;
    void *keys = w->keys;
    auto dst = [stage](int64_t, int64_t) { return stage; };
    auto after = [&](int64_t r0, int64_t nr, const void *dev) -> int {
        dim3 grid((unsigned)((nr + 31) / 32), (unsigned)((p + 31) / 32));
        if (dtype)
            k_keys<double><<<grid, 256, 0, st>>>(static_cast<const double *>(dev), nr, p, r0, n,
                                                 static_cast<unsigned long long *>(keys));
        else
            k_keys<float><<<grid, 256, 0, st>>>(static_cast<const float *>(dev), nr, p, r0, n,
                                                static_cast<uint32_t *>(keys));
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? 0 : cuda_fail(err, "k_keys", e);
    };
    if (gbmh2d::stream_rows(sg, st, X, n, row, gbmh2d::Pack::Copy, 0, dst, after, err)) {
        w->dtype = -1;
        return -1;
    }
    return 0;
}

namespace {

template <typename T>
int edges_t(Work *w, cudaStream_t st, int n_bins, const std::vector<uint8_t> &skip, int stride, double *h_edges,
            int32_t *h_counts, int32_t *h_nanb, std::string &err) {
    typedef typename Keys<T>::K K;
    const int64_t n = w->n;
    const int p = w->p;
    const int cap = n_bins + 1;
    if (ensure(&w->sorted, w->sorted_cap, (size_t)n * p * sizeof(K), err)) return -1;
    // per-feature arrays: nclean (8) nuniq (4) skip (1) counts (4) nanb (4),
    // uq [p][cap], edges [p][stride], the two quantile tables
    std::vector<double> qa, qn;
    quantiles(n_bins + 1, qa);
    quantiles(n_bins, qn);
    const size_t o_nc = 0;
    const size_t o_nu = o_nc + 8 * (size_t)p;
    const size_t o_cnt = o_nu + 4 * (size_t)p;
    const size_t o_nb = o_cnt + 4 * (size_t)p;
    const size_t o_skip = o_nb + 4 * (size_t)p;
    const size_t o_uq = (o_skip + (size_t)p + 15) & ~(size_t)15;
    const size_t o_ed = o_uq + 8 * (size_t)p * cap;
    const size_t o_qa = o_ed + 8 * (size_t)p * stride;
    const size_t o_qn = o_qa + 8 * qa.size();
    const size_t total = o_qn + 8 * qn.size();
    if (ensure(&w->small, w->small_cap, total, err)) return -1;
    char *sm = static_cast<char *>(w->small);
    long long *d_nc = reinterpret_cast<long long *>(sm + o_nc);
    int *d_nu = reinterpret_cast<int *>(sm + o_nu);
    int *d_cnt = reinterpret_cast<int *>(sm + o_cnt);
    int *d_nb = reinterpret_cast<int *>(sm + o_nb);
    uint8_t *d_skip = reinterpret_cast<uint8_t *>(sm + o_skip);
    double *d_uq = reinterpret_cast<double *>(sm + o_uq);
    double *d_ed = reinterpret_cast<double *>(sm + o_ed);
    double *d_qa = reinterpret_cast<double *>(sm + o_qa);
    double *d_qn = reinterpret_cast<double *>(sm + o_qn);
    BCK("edges tables", cudaMemcpyAsync(d_skip, skip.data(), (size_t)p, cudaMemcpyHostToDevice, st));
    BCK("edges tables", cudaMemcpyAsync(d_qa, qa.data(), 8 * qa.size(), cudaMemcpyHostToDevice, st));
    BCK("edges tables", cudaMemcpyAsync(d_qn, qn.data(), 8 * qn.size(), cudaMemcpyHostToDevice, st));
    const K *keys = static_cast<const K *>(w->keys);
    K *sorted = static_cast<K *>(w->sorted);
    size_t tmp_bytes = 0;
    BCK("radix sort", cub::DeviceRadixSort::SortKeys(nullptr, tmp_bytes, keys, sorted, (int)n, 0, Keys<T>::kBits, st));
    if (ensure(&w->tmp, w->tmp_cap, tmp_bytes, err)) return -1;
    for (int j = 0; j < p; j++) {
        if (skip[(size_t)j]) continue;
        size_t tb = w->tmp_cap;
        BCK("radix sort", cub::DeviceRadixSort::SortKeys(w->tmp, tb, keys + (int64_t)j * n, sorted + (int64_t)j * n,
                                                         (int)n, 0, Keys<T>::kBits, st));
    }
    k_edge_scan<T><<<p, kScanThreads, 0, st>>>(sorted, n, d_skip, n_bins, cap, d_nc, d_nu, d_uq);
    BCK("k_edge_scan", cudaGetLastError());
    k_edge_final<T><<<p, kFinalThreads, 0, st>>>(sorted, n, d_skip, n_bins, cap, d_nc, d_nu, d_uq, d_qa, d_qn, d_ed,
                                                stride, d_cnt, d_nb);
    BCK("k_edge_final", cudaGetLastError());
    BCK("edges copy", cudaMemcpyAsync(h_edges, d_ed, 8 * (size_t)p * stride, cudaMemcpyDeviceToHost, st));
    BCK("edges copy", cudaMemcpyAsync(h_counts, d_cnt, 4 * (size_t)p, cudaMemcpyDeviceToHost, st));
    BCK("edges copy", cudaMemcpyAsync(h_nanb, d_nb, 4 * (size_t)p, cudaMemcpyDeviceToHost, st));
    BCK("edges", cudaStreamSynchronize(st));
    return 0;
}

// Uploads edges/counts/NaN bins for the binning kernels; returns the table
// size (a power of two >= every bin count) or -1.
int stage_tables(Work *w, cudaStream_t st, int p, const double *edges, int stride, const int32_t *counts,
                 const int32_t *nan_bin, double **d_ed, int **d_cnt, int **d_nb, int &any_nan, std::string &err) {
    int maxc = 1;
    any_nan = 0;
    for (int j = 0; j < p; j++) {
        if (counts[j] < 1 || counts[j] >= stride || counts[j] > kMaxTab) {
            char buf[160];
            snprintf(buf, sizeof buf, "binning: feature %d has %d bins (1..%d and below the edge stride %d)", j,
                     counts[j], kMaxTab, stride);
            err = buf;
            return -1;
        }
        maxc = std::max(maxc, (int)counts[j]);
        any_nan |= nan_bin[j] >= 0;
    }
    const size_t o_ed = 0, o_cnt = 8 * (size_t)p * stride, o_nb = o_cnt + 4 * (size_t)p;
    if (ensure(&w->small, w->small_cap, o_nb + 4 * (size_t)p, err)) return -1;
    char *sm = static_cast<char *>(w->small);
    *d_ed = reinterpret_cast<double *>(sm + o_ed);
    *d_cnt = reinterpret_cast<int *>(sm + o_cnt);
    *d_nb = reinterpret_cast<int *>(sm + o_nb);
    BCK("bin tables", cudaMemcpyAsync(*d_ed, edges, 8 * (size_t)p * stride, cudaMemcpyHostToDevice, st));
    BCK("bin tables", cudaMemcpyAsync(*d_cnt, counts, 4 * (size_t)p, cudaMemcpyHostToDevice, st));
    BCK("bin tables", cudaMemcpyAsync(*d_nb, nan_bin, 4 * (size_t)p, cudaMemcpyHostToDevice, st));
    return next_pow2(maxc);
}

template <typename F>
void smem_opt_in(F kernel, size_t bytes) {
    if (bytes > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

unsigned bin_grid_x(int64_t rows, int nblk) {
    const int64_t want = (rows + kBinThreads - 1) / kBinThreads;
    const int64_t cap = std::max<int64_t>(1, 148 * 8 / std::max(1, nblk));
    return (unsigned)std::max<int64_t>(1, std::min(want, cap));
}

}  // namespace

int edges(Work *w, cudaStream_t st, int n_bins, const uint8_t *is_cat, double *edges_out, int stride,
          int32_t *counts_out, int32_t *nan_bin_out, int32_t *max_b_out, std::string &err) {
    if (w->dtype < 0) {
        err = "binning: no matrix loaded";
        return -1;
    }
    if (n_bins < 2 || n_bins > kMaxBins) {
        err = "binning: n_bins must be in 2..1023";
        return -1;
    }
    if (stride < std::max(n_bins + 2, 65)) {
        err = "binning: edge stride must be at least max(n_bins + 2, 65)";
        return -1;
    }
    if (!edges_out || !counts_out || !nan_bin_out) {
        err = "binning: null output";
        return -1;
    }
    const int p = w->p;
    std::vector<uint8_t> skip((size_t)p, 0);
    if (is_cat)
        for (int j = 0; j < p; j++) skip[(size_t)j] = is_cat[j] != 0;
    const int rc = w->dtype ? edges_t<double>(w, st, n_bins, skip, stride, edges_out, counts_out, nan_bin_out, err)
                            : edges_t<float>(w, st, n_bins, skip, stride, edges_out, counts_out, nan_bin_out, err);
    if (rc) return rc;
    int maxc = 0;
    for (int j = 0; j < p; j++) {
        if (skip[(size_t)j]) {   // exact integer bins 0..63 (E:2086-2090)
            double *row = edges_out + (size_t)j * stride;
            for (int t = 0; t < stride; t++) row[t] = -0.5 + (double)std::min(t, 64) * 1.0;
            counts_out[j] = 64;
            nan_bin_out[j] = -1;
        }
        maxc = std::max(maxc, (int)counts_out[j]);
    }
    if (max_b_out) *max_b_out = maxc + 1;
    return 0;
}

int bin_blocks(Work *w, cudaStream_t st, int64_t lo, int64_t hi, const double *edges, int stride,
               const int32_t *counts, const int32_t *nan_bin, uint8_t *d_xb, const int32_t *d_bigidx,
               uint32_t *d_topbits, std::string &err) {
    if (w->dtype < 0) {
        err = "binning: no matrix loaded";
        return -1;
    }
    if (lo < 0 || hi > w->n || hi <= lo) {
        err = "binning: bad row range";
        return -1;
    }
    const int p = w->p;
    double *d_ed;
    int *d_cnt, *d_nb, any_nan;
    const int ts = stage_tables(w, st, p, edges, stride, counts, nan_bin, &d_ed, &d_cnt, &d_nb, any_nan, err);
    if (ts < 0) return -1;
    const int nblk = (p + 15) / 16;
    const int64_t rows = hi - lo;
    dim3 grid(bin_grid_x(rows, nblk), (unsigned)nblk);
    if (w->dtype) {
        const size_t sm = 16 * (size_t)ts * sizeof(double);
        smem_opt_in(k_bin_keys<double>, sm);
        k_bin_keys<double><<<grid, kBinThreads, sm, st>>>(static_cast<const unsigned long long *>(w->keys), w->n, p,
                                                          lo, rows, d_ed, stride, d_cnt, d_nb, any_nan, ts, d_xb,
                                                          d_bigidx, d_topbits);
    } else {
        const size_t sm = 16 * (size_t)ts * sizeof(float);
        smem_opt_in(k_bin_keys<float>, sm);
        k_bin_keys<float><<<grid, kBinThreads, sm, st>>>(static_cast<const uint32_t *>(w->keys), w->n, p, lo, rows,
                                                         d_ed, stride, d_cnt, d_nb, any_nan, ts, d_xb,
                                                         d_bigidx, d_topbits);
    }
    BCK("k_bin_keys", cudaGetLastError());
    return 0;
}

int bin_rows(Work *w, gbmh2d::Stager *sg, cudaStream_t st, const void *X, int64_t n, int p, int dtype,
             const double *edges, int stride, const int32_t *counts, const int32_t *nan_bin, int out_mode, void *out,
             const int32_t *d_bigidx, uint32_t *d_topbits, std::string &err) {
    if (!X || !out || n <= 0 || p <= 0 || (dtype != 0 && dtype != 1) || (out_mode != 0 && out_mode != 1)) {
        err = "binning: bad arguments";
        return -1;
    }
    const size_t ts_bytes = dtype ? 8 : 4;
    const size_t row = (size_t)p * ts_bytes;
    if (row > gbmh2d::chunk_bytes()) {
        err = "binning: rows wider than the upload buffers";
        return -1;
    }
    double *d_ed;
    int *d_cnt, *d_nb, any_nan;
    const int ts = stage_tables(w, st, p, edges, stride, counts, nan_bin, &d_ed, &d_cnt, &d_nb, any_nan, err);
    if (ts < 0) return -1;
    if (ensure(&w->stage, w->stage_cap, gbmh2d::chunk_bytes(), err)) return -1;
    const int64_t chunk_rows = (int64_t)(gbmh2d::chunk_bytes() / row);
    if (out_mode == 1 && ensure(&w->ostage, w->ostage_cap, (size_t)chunk_rows * p * 2, err)) return -1;
    const int nblk = (p + 15) / 16;
    const size_t sm = 16 * (size_t)ts * (dtype ? sizeof(double) : sizeof(float));
    if (dtype) {
        smem_opt_in(k_bin_rows<double, 0>, sm);
        smem_opt_in(k_bin_rows<double, 1>, sm);
    } else {
        smem_opt_in(k_bin_rows<float, 0>, sm);
        smem_opt_in(k_bin_rows<float, 1>, sm);
    }
    void *stage = w->stage;
    void *ostage = w->ostage;
    auto dst = [stage](int64_t, int64_t) { return stage; };
    auto after = [&](int64_t r0, int64_t nr, const void *dev) -> int {
        dim3 grid(bin_grid_x(nr, nblk), (unsigned)nblk);
        void *o = out_mode == 0 ? static_cast<void *>(static_cast<uint8_t *>(out) + (size_t)r0 * p) : ostage;
        if (dtype) {
            if (out_mode == 0)
                k_bin_rows<double, 0><<<grid, kBinThreads, sm, st>>>(static_cast<const double *>(dev), nr, p, d_ed,
                                                                     stride, d_cnt, d_nb, any_nan, ts, o, d_bigidx, d_topbits, r0, (n + 31) >> 5);
            else
                k_bin_rows<double, 1><<<grid, kBinThreads, sm, st>>>(static_cast<const double *>(dev), nr, p, d_ed,
                                                                     stride, d_cnt, d_nb, any_nan, ts, o, d_bigidx, d_topbits, r0, (n + 31) >> 5);
        } else {
            if (out_mode == 0)
                k_bin_rows<float, 0><<<grid, kBinThreads, sm, st>>>(static_cast<const float *>(dev), nr, p, d_ed,
                                                                    stride, d_cnt, d_nb, any_nan, ts, o, d_bigidx, d_topbits, r0, (n + 31) >> 5);
            else
                k_bin_rows<float, 1><<<grid, kBinThreads, sm, st>>>(static_cast<const float *>(dev), nr, p, d_ed,
                                                                    stride, d_cnt, d_nb, any_nan, ts, o, d_bigidx, d_topbits, r0, (n + 31) >> 5);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(err, "k_bin_rows", e);
        if (out_mode == 1) {
            e = cudaMemcpyAsync(static_cast<uint16_t *>(out) + (size_t)r0 * p, ostage, (size_t)nr * p * 2,
                                cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) return cuda_fail(err, "bin ids copy", e);
        }
        return 0;
    };
    if (gbmh2d::stream_rows(sg, st, X, n, row, gbmh2d::Pack::Copy, chunk_rows, dst, after, err)) return -1;
    return 0;
}

}  // namespace gbmbin
