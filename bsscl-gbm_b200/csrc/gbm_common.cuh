// gbm_common.cuh -- constants, device helpers and the structures shared by
// the engine's kernels (gbm_kernels.cuh) and its host code (gbm_b200.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

namespace gbm {

constexpr int kBins = 256;          // uint8 bin ids
constexpr int kBlk = 16;            // features per column block (one 16-byte load)
constexpr int kWords = 4;           // g_hi, g_lo, h_hi, h_lo per histogram cell
constexpr int kTotWords = 6;        // after the cells: totals (G hi/lo, H hi/lo), left count, pad
constexpr int kCountWord = 4;       // the slot's left-count word (multi-rank staging)
// The fixed-point exponent: S = 62 - ceil(log2(kChunk * max(1, w_max))), so
// |q| <= 2^48 for every row and 2^15 rows of q sum to less than 2^63.
constexpr int kChunk = 16384;
constexpr int kDig = 17;            // low/mid digit width of the shared-memory accumulators
constexpr int kRowWeight = 6 + kBlk;     // k_hist3's cost of a row of a block (its loads + 16 steps)
constexpr int kPartTile = 4096;     // rows per partition CTA
constexpr int kPartThreads = 512;   // 8 rows per thread, loads in flight together
constexpr int kPartWords = kPartTile / 32;   // side bits of a tile
constexpr int kUpdThreads = 256;
constexpr int kCompTile = 4096;     // rows per in-bag compaction CTA

typedef __int128 i128;

// A histogram slot: [nf][256] cells of kWords, the node's kTotWords total
// words, then one more cell per feature position -- the top cell, the sum
// over the rows whose bin id is 256 (features with 257 bins: stored as 255,
// see top_cell_offset).
__host__ __device__ __forceinline__ int64_t slot_words_for(int nf) {
    return (int64_t)nf * kBins * kWords + kTotWords + (int64_t)nf * kWords;
}

// Word offset of feature position jj's top cell in a slot.  A feature with
// 257 bins (ids 0..256: n_bins 256, E:2111-2127) is stored with ids
// min(id, 255), so its cell 255 holds bins 255 and 256 together, and this
// cell holds bin 256 alone (the rows equal to the column maximum); every
// threshold 0..255 of the reference's scan is then exact.
__host__ __device__ __forceinline__ int64_t top_cell_offset(int nf, int jj) {
    return (int64_t)nf * kBins * kWords + kTotWords + (int64_t)jj * kWords;
}

// Row r's bit of a top-bin matrix (bits [big feature][ceil(n / 32)] words):
// 1 when its bin id is 256.
__device__ __forceinline__ bool top_bit(const uint32_t *__restrict__ bits, int64_t words_per, int big, int64_t r) {
    return big >= 0 && bits && ((__ldg(bits + (int64_t)big * words_per + (r >> 5)) >> (r & 31)) & 1u);
}

// ---------------------------------------------------------------------------
// structures
// ---------------------------------------------------------------------------

// One node of the tree being grown, as known to the device.  Histogram
// slot of node i is pool slot i.
struct DNode {
    long long begin, end;   // this rank's rows: rows[begin, end)
    long long n;            // rows over all ranks
    long long nl, gnl;      // rows sent left (this rank / all ranks) once expanded
    double G, H;            // exact totals, each rounded once to float64
    double gain;            // best split gain (meaningful when feat >= 0)
    int feat, bin;          // best split; feat = -1: none, or the node may not split
    int depth, parent;
    int kid0, kid1;         // children (-1 = not expanded)
    int left_small;         // 1 if the left child's histogram was built directly
    int expanded;           // 1 once both children's results are final
    int nan_right;          // the best split sends the NaN bin (bin 0) right (learned direction)
    int pad;
    double mg;              // best-first pruning: the smallest gain on the path of valid splits from
                            // the root to this node, -inf when the path holds a split that cannot be made
};

// Row lists live in two buffers: the rows of a node at depth d are in
// buffer d & 1, and a partition writes the children into the other one.
struct HistTask {           // rows[buf][begin, end) -> staging histogram `stage`
    long long begin, end;
    int stage;
    int left_small;
    int buf;
    int pad;
};

struct PartTask {           // stable partition of rows[src][begin, end) on goes_left(bin(feat), thr, nan_right)
    long long begin, end;
    int feat, thr;
    int tile0, ntile;       // tiles of this task in the level's tile numbering
    int src;                // the parent's buffer; the children go to 1 - src
    int nan_right;
};

struct FBest {              // best bin of one feature for one node
    double gain;
    int bin;
    int valid;
    int nan_right;          // the best candidate sends the NaN bin right
    int pad;
};

struct TreeDev {            // a pruned tree in the reference's layout
    int n;
    int feat[256];
    int thr[256];           // threshold bin (<= 255) | nan_right << 16 (dev_thr)
    int left[256];
    int right[256];
    double val[256];
};

// One finished tree in the reference's tuple layout, written by the device
// replay and copied to the host.
struct TreeOut {
    int nc;
    int status;             // 0 ok, 1 the replay needed a node that was not expanded, 3 a partition wait ran out
    long long root_rows;    // this rank's in-bag rows
    long long alg_rows;     // root rows + the smaller child's rows of every split (this rank)
    int tf[256];
    int tl[256];
    int tr[256];
    long long tt[256];
    double tv[256];
    double sg[256];
    int nr[256];            // 1: the split sends the NaN bin right (learned direction)
};

struct RParams {            // growth parameters the replay needs
    double lam, gamma, mcw;
    long long msl;
    int max_depth, max_leaves, policy, has_mono;
    const int *part_err;    // set by a partition look-back wait that ran out (the tree's status 3)
};

struct PNode {              // predict: 8 bytes per node
    int16_t feat;           // -1 = leaf
    uint8_t thr;
    uint8_t nanr;           // bit 0: the NaN bin (bin 0) goes right; bit 1: the threshold is above
                            // 255 (stored 255), so bin 256 of a 257-bin feature goes left too
    int16_t left, right;    // tree-local ids
};

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

// A histogram cell stores a 128-bit sum as two int64 words: hi * 2^32 + lo.
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

__device__ __forceinline__ i128 shfl_up_i128(i128 v, int o) {
    long long lo = (long long)(unsigned long long)v;
    long long hi = (long long)(v >> 64);
    lo = __shfl_up_sync(0xffffffffu, lo, o);
    hi = __shfl_up_sync(0xffffffffu, hi, o);
    return ((i128)hi << 64) | (i128)(unsigned long long)lo;
}

__device__ __forceinline__ i128 shfl_xor_i128(i128 v, int m) {
    long long lo = (long long)(unsigned long long)v;
    long long hi = (long long)(v >> 64);
    lo = __shfl_xor_sync(0xffffffffu, lo, m);
    hi = __shfl_xor_sync(0xffffffffu, hi, m);
    return ((i128)hi << 64) | (i128)(unsigned long long)lo;
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

__device__ __forceinline__ int bin_of(const uint8_t *__restrict__ xb, int64_t n, int64_t row, int f) {
    return __ldg(xb + (((int64_t)(f >> 4) * n + row) << 4) + (f & 15));
}

// Throughput-mode row sampling (gbm_sampler_create_device): row `row`
// (global id) is in-bag in round `round` iff this hash is below the
// sampler's threshold.  The mixing is the splitmix64 finalizer (Steele, Lea
// and Flood, 2014) of seed + round * k1 + row * k2; every rank hashes its own
// rows, so the draw is the same at any GPU count and needs no exchange.
__host__ __device__ __forceinline__ uint64_t gbm_row_hash(uint64_t seed, uint64_t round, uint64_t row) {
    uint64_t z = seed + round * 0xd1b54a32d192ed03ull + row * 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// The split rule.  The reference sends bin <= thr left (E:668, E:855,
// E:878), so the NaN bin (bin 0) always goes left.  A split learned with the
// NaN direction (gbm_params.nan_direction) may instead send the NaN bin
// right: then left is 1 <= bin <= thr (thr >= 1).
__host__ __device__ __forceinline__ bool goes_left(int b, int thr, int nan_right) {
    return b <= thr && !(nan_right && b == 0);
}

// A tree threshold as the update kernels read it: the bin (clamped to 255)
// with the NaN direction in bit 16.
__host__ __device__ __forceinline__ int dev_thr(long long t, int nan_right) {
    return (int)(t > 255 ? 255 : t) | (nan_right ? 1 << 16 : 0);
}

// a beats b: larger gain; equal gains -> lower feature position, then lower bin
// (the reference's strict '>' scan over ascending features and bins).
__device__ __forceinline__ bool better(double ga, int ja, int ba, double gb, int jb, int bb) {
    if (ja < 0) return false;
    if (jb < 0) return true;
    if (ga > gb) return true;
    if (gb > ga) return false;
    if (ja != jb) return ja < jb;
    return ba < bb;
}

}  // namespace gbm
