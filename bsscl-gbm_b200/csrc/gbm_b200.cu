// gbm_b200.cu -- host side of the B200 engine: context, tree growth, the
// best-first replay, and the C ABI (include/gbm_b200.h).
//
// One boosting round of HybridHistGBMNumbaV1_0_1._fit_binary
// (src/bsscl_gbm/estimator_v1_0_1.py, "E" below, E:2849-2905):
//
//   1. in-bag rows -> ascending row list (mask compaction);
//   2. the tree is grown level by level on the device with no host round
//      trip: the root histogram and split, then per level every parent in
//      the level list is partitioned (E:663-674), the smaller child's
//      histogram is built (E:723-737), the larger one is parent - smaller
//      (E:740-745), and both children's best splits are searched
//      (E:775-801); the next level list is the children with a split,
//      ranked by gain and capped (speculation: a node may be expanded that
//      best-first never splits -- its result is simply unused);
//   3. the host fetches the node table once and replays the reference's
//      best-first selection exactly (E:642-823: candidate slots, strict '>'
//      with lowest slot winning, min_samples_leaf on the partition, node
//      numbering); a node the replay needs that was not expanded is
//      expanded on demand (same device level machinery, host-made list);
//   4. post-prune (E:827-841), monotone clipping (E:2461-2499), then one
//      kernel updates F, the logloss and the next round's gradients.
//
// Exactness.  Every g and h is rounded once to the grid 2^-S and all sums
// are integer sums, so every histogram, total and gain is independent of
// row order, CTA schedule and GPU count (gbm_kernels.cuh has the details).

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <string>
#include <utility>
#include <vector>

#include "../../include/gbm_b200.h"
#include "binning_internal.h"
#include "comm.h"
#include "h2d.h"
#include "sampler_internal.h"
#include "gbm_kernels.cuh"

using namespace gbm;

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
    // the round's selected features packed in blocks of 16 (k_compact_feat):
    // two buffers, round r uses [slot & 1], so the sampler stream can pack
    // round r + 1 while round r's histograms read the other
    uint8_t *d_xc[2] = {nullptr, nullptr};
    const uint8_t *xc_cur = nullptr;   // the buffer of the round being enqueued
    int32_t *d_counts = nullptr;
    std::vector<int32_t> counts;
    // Features with 257 bins (ids 0..256, n_bins 256: E:2111-2127) keep
    // min(id, 255) in d_xb; the rows whose id is 256 are bits of d_topbits
    // [nbig][ceil(n / 32)] and, as ascending row lists, d_toprows
    // [d_topoff[b] .. d_topoff[b + 1]).  d_bigidx [p]: the feature's index
    // among them, -1 for every other feature.
    int nbig = 0;
    std::vector<int32_t> bigfeat;
    int32_t *d_bigidx = nullptr, *d_bigfeat = nullptr, *d_topoff = nullptr, *d_toprows = nullptr;
    uint32_t *d_topbits = nullptr;
    int64_t *d_toppairs = nullptr;   // the uint16 upload's (row, big index) pairs of id 256
    uint8_t *d_y = nullptr;
    double *d_F = nullptr;
    longlong2 *d_q = nullptr;
    double w[2] = {1.0, 1.0};
    double base = 0.0;
    int S = 0;
    bool have_bins = false, have_labels = false;

    // round buffers
    // The round's in-bag mask, its two row-list buffers (depth parity) and
    // its compaction scratch: aliases of one of two sets, by round parity
    // (slot & 1), so the sampler stream builds round r + 1's root list
    // while round r still partitions its own.
    uint8_t *d_mask = nullptr;
    int32_t *d_rows = nullptr, *d_tmp = nullptr;
    uint8_t *d_maskP[2] = {};
    int32_t *d_rowsP[2] = {}, *d_tmpP[2] = {}, *d_totalP[2] = {};
    unsigned long long *d_compP[2] = {};   // k_compact_rows' tile words, then its [ticket, done]
    cudaEvent_t rows_freeP[2] = {};
    unsigned long long *d_tile_st = nullptr;       // k_partition's per-tile look-back words (zero between levels)
    int32_t *d_total = nullptr;
    unsigned long long *d_comp = nullptr;
    int32_t *d_blist = nullptr, *d_fidx = nullptr;
    int16_t *d_fpos = nullptr, *d_fbi = nullptr;
    int hist_grid = 0;                 // 2 CTAs per SM: the grid of the multi-rank staging kernels
    int sms = 0;
    // Histogram launches of a tree, from the root, that use k_hist2 (big
    // segments: its conflict-free atomics win); the deeper, smaller
    // segments use k_hist, whose two CTAs per SM overlap one CTA's zeroing
    // and flush with the other's atomics.  Measured on config 4: 3 levels
    // 1110 rounds/s, 0 levels 1077, all levels 1057.
    bool hist_compact = true;          // histograms on the round's packed feature blocks (k_compact_feat)
    int hist_seg_cost = 150000;        // k_hist3's cost of a segment in row units (22 per row; measured)
    int nf_cap = 0;
    long long *d_pool = nullptr;       // node histograms: slot i = node i
    long long *d_lpool = nullptr;      // several ranks: this rank's partial histograms, slot i = node i
    int64_t lpool_words = 0;
    // Several ranks, peer exchange of the staging slots over NVLink (CUDA IPC;
    // gbm_kernels.cuh, "the staging exchange").  Off: one NCCL all-reduce per level.
    bool p2p = false;
    int64_t p2p_tried_stride = 0;      // the staging size the last setup was made for
    int p2p_rank = 0, p2p_n = 1;
    long long *d_pst = nullptr;        // two parity buffers of stage_slots slots (IPC-exported)
    int64_t pst_stride = 0;            // words per parity buffer
    unsigned long long *d_sync = nullptr;   // signals from each rank and local words (IPC-exported)
    long long *d_red = nullptr;        // two-shot exchange: this rank's summed share of a level (IPC-exported)
    long long **d_peer_pst = nullptr;       // every rank's d_pst (own at [rank]), device table
    long long **d_peer_red = nullptr;       // every rank's d_red
    unsigned long long **d_peer_sync = nullptr;
    std::vector<void *> ipc_opened;    // peer mappings to close
    long long *d_stage = nullptr;      // smaller-child histograms of one level
    int stage_slots = 0;
    int nmax = 0;                      // node capacity of the tree table
    FBest *d_fbest = nullptr;
    HistTask *d_htask = nullptr;
    int32_t *d_hprefix = nullptr;
    PartTask *d_ptask = nullptr;
    int tile_cap = 0;
    long long *d_nleft = nullptr, *d_count64 = nullptr;   // d_count64: one word for small all-reduces
    long long *d_leafw = nullptr;      // last level: per-parent count and (G, H) words
    DNode *d_nodes = nullptr;
    int *d_lvl[2] = {nullptr, nullptr};
    int *d_ints = nullptr;             // [0] one, [1] node count, [2] tiles, [3..4] level counts
    TreeDev *d_tree = nullptr;
    int32_t *d_leaf = nullptr;
    double *d_loss_part = nullptr, *d_loss = nullptr;
    int upd_blocks = 0;
    // pinned host mirrors
    DNode *h_nodes = nullptr;
    TreeOut *h_tout_mc = nullptr;   // multi-class rounds: one tree record per class
    int *h_ints = nullptr;
    int *h_list = nullptr;
    double *h_loss = nullptr;
    uint8_t *h_mask = nullptr;
    std::vector<int32_t> feat_buf;

    // Rounds in flight: per-slot pinned staging (so no copy waits for the
    // stream) and a completion event.  gbm_round* use slot 0 and wait at the
    // end; gbm_fit_rounds keeps up to kRing rounds queued.
    struct Slot {
        int32_t *h_tg = nullptr, *d_tg = nullptr;   // the round's row swap targets
        long long *h_round = nullptr, *d_round = nullptr;   // the round's index (throughput-mode rows)
        int32_t *h_feat = nullptr;     // fidx [p] | blist [nblk] | nb
        int32_t *d_fidx_c = nullptr;   // the round's fidx for its feature compaction on cst
        bool xc_on_cst = false;        // the round's packed blocks are made on cst (k_compact_feat)
        int16_t *h_fpos = nullptr;     // fpos [nblk * 16] | fbi [p]
        TreeOut *h_tout = nullptr;
        double *h_loss = nullptr;
        double upd_per_row = 0.0;      // histogram cell updates per row of this round
        cudaEvent_t copied = nullptr, done = nullptr;
        // timing pairs recorded by this slot's round while profiling (kind 0:
        // k_hist, 1: L2 flush); a captured round records the same pairs every run
        std::vector<cudaEvent_t> tev;
        std::vector<char> tkind;
        int tused = 0, tdone = 0;
        // the slot's captured round (gbm_fit_rounds)
        cudaGraphExec_t g_cst = nullptr, g_st = nullptr;
        int g_tpairs = 0;
        long long g_launches = 0, g_hist = 0, g_waves = 0;
        double g_comm_bytes = 0.0;
    };
    static constexpr int kRing = 4;
    Slot slot[kRing];
    bool slots_ready = false;
    cudaStream_t cst = nullptr;        // the samplers' copies, row shuffles and root row lists
    cudaEvent_t rows_free = nullptr;   // recorded on st once a round is done with its row lists (alias by parity)
    int cur_slot = 0;                  // the slot whose round is being enqueued
    bool capturing = false;            // enqueueing into a graph capture
    std::string graph_key;             // what the slots' graphs were captured for
    unsigned long long mem_gen = 0;    // bumped by every (re)allocation: graphs hold pointers
    // The bound sampler's row permutation lives here: round r turns its swap
    // targets into a shuffle and composes perm[r % 5] = perm[(r-1) % 5][S]
    // on cst, ahead of the round's growth.
    gbm_sampler *samp = nullptr;
    int64_t samp_taken = 0;
    int64_t shuf_n = 0;
    int32_t *d_perm[kRing] = {};
    int32_t *d_head = nullptr, *d_nxt = nullptr, *d_m = nullptr, *d_mp = nullptr;
    TreeOut *d_tout = nullptr;
    int32_t *d_mono = nullptr, *h_mono = nullptr;
    uint8_t *d_nanf = nullptr, *h_nanf = nullptr;   // per feature: bin 0 is a NaN bin (nan_direction)
    bool nan_dir = false;                           // this call's rounds learn the NaN direction
    int replay_smem = 0;               // dynamic shared memory the replay kernels may use

    // regression: float64 targets, mse (0) or mae (1); S follows the largest |g| each round
    bool have_targets = false;
    int reg_mae = 0;
    double *d_yr = nullptr, *d_gmax_part = nullptr, *d_gmax = nullptr;
    long long *d_stab = nullptr;       // several ranks: the one-hot table of the proposed S
    // multi-class softmax: K classes, F and q class-major ([k][n])
    int K = 0;
    bool have_labels_mc = false;
    double *d_Fmc = nullptr, *d_wmc = nullptr;
    longlong2 *d_qmc = nullptr;

    // predict
    uint8_t *d_px = nullptr;
    int64_t pn = 0, pn_cap = 0;
    int32_t pp = 0;
    uint8_t *d_pnodes = nullptr;    // PNode [total], or the 32-bit breadth-first words when p_packed
    bool p_packed = false;
    bool p_packed_nr = false;       // the packed words hold NaN-right splits
    double *d_pvals = nullptr;
    int32_t *d_poff = nullptr;
    int4 *d_pchunk = nullptr;       // [p_trees_cap] chunks of whole trees, then the chunk count
    int32_t *d_pdep = nullptr;      // [p_trees_cap] tree depths (the packed format)
    int32_t p_ntree = 0;
    int64_t p_nodes_cap = 0;
    int32_t p_trees_cap = 0;
    int32_t p_nfeat = 0;
    double *d_pF = nullptr, *d_pP = nullptr;
    // the predict rows' bin-256 bits, as for training (null when no feature has them)
    int32_t *d_pbigidx = nullptr;
    uint32_t *d_ptopbits = nullptr;
    bool p_top = false;
    bool p_model_top = false;   // the model has a threshold of 255 (the bits matter)

    // uploads and binning
    gbmh2d::Stager *stager = nullptr;  // pinned ring + copy threads for host -> device streams
    uint8_t *d_upstage = nullptr;      // device side of one upload chunk
    gbmbin::Work *bw = nullptr;        // the raw matrix as order keys, sort buffers, tables

    // instrumentation
    long long launches = 0;          // every kernel this context launched
    bool profiling = false;
    long long hist_launches = 0, hist_rows = 0, waves = 0;
    double hist_ms = 0.0, alg_bytes = 0.0, hist_updates = 0.0;
    double host_sample_ms = 0.0, host_sync_ms = 0.0, host_replay_ms = 0.0, host_comm_ms = 0.0;
    double comm_ms = 0.0, comm_bytes = 0.0;   // collectives: device time (profiling), bytes per rank
    double peer_wait_base_ms = 0.0;           // the peer exchange's wait counter at the last stats reset
    // benchmark aid: an L2 eviction at the start of every round
    uint8_t *d_flush = nullptr;
    size_t flush_bytes = 0;
    unsigned flush_count = 0;
    double flush_ms = 0.0;
    double samp_ms = 0.0, samp_stall_ms = 0.0;   // profiling: timing pairs of kinds 3 and 4

    cudaEvent_t mark[16] = {};
    std::unordered_map<void *, size_t> dcap, hcap;   // bytes of each buffer dalloc / halloc made
};

namespace {

// d_ints: I_DONE / I_DONE_UPD / I_DONE_LEAF count finished CTAs of
// k_partition / k_update / k_leaf_totals (the last one runs the tail and
// resets it); I_TICKET hands out k_partition's tiles in order; I_PART_ERR
// records a partition look-back wait that ran out
enum { I_ONE = 0, I_NODES = 1, I_TILES = 2, I_LVL0 = 3, I_LVL1 = 4, I_DONE = 5, I_DONE_UPD = 6, I_TICKET = 7,
       I_PART_ERR = 8, I_DONE_LEAF = 9, I_COUNT = 10 };

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

// Kernels of a round are launched with programmatic stream serialization:
// a kernel may be scheduled while its predecessor drains, and it waits
// (griddep_wait, its first statement) before reading anything the
// predecessor wrote.  That hides most of the gap between dependent launches.
template <typename... P, typename... A>
int launch(gbm_ctx *ctx, void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A &&...args) {
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    ctx->launches++;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
    if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
    return GBM_OK;
}

// Event record / wait that also work inside a graph capture, where they
// become event nodes recorded or waited on at every run of the graph.
int record_ev(gbm_ctx *ctx, cudaEvent_t ev, cudaStream_t s) {
    cudaError_t e = ctx->capturing ? cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal) : cudaEventRecord(ev, s);
    if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "event record: %s", cudaGetErrorString(e));
    return GBM_OK;
}

int wait_ev(gbm_ctx *ctx, cudaStream_t s, cudaEvent_t ev) {
    cudaError_t e = cudaStreamWaitEvent(s, ev, ctx->capturing ? cudaEventWaitExternal : 0);
    if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "event wait: %s", cudaGetErrorString(e));
    return GBM_OK;
}

// A timing pair (start, end) of the current slot's round; kind 0: k_hist,
// 1: the L2 flush, 2: a collective, 3: the round's sampler-stream work, 4: the
// engine stream's wait for it.
int timing_pair(gbm_ctx *ctx, char kind, cudaEvent_t &e0, cudaEvent_t &e1) {
    gbm_ctx::Slot &s = ctx->slot[ctx->cur_slot];
    while ((int)s.tev.size() < 2 * (s.tused + 1)) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        s.tev.push_back(e);
    }
    if ((int)s.tkind.size() < s.tused + 1) s.tkind.resize((size_t)s.tused + 1);
    s.tkind[(size_t)s.tused] = kind;
    e0 = s.tev[(size_t)(2 * s.tused)];
    e1 = s.tev[(size_t)(2 * s.tused + 1)];
    s.tused++;
    return GBM_OK;
}

// The engine stream waits for the slot's sampler-stream work (profiling:
// timed as kind 4).
int wait_copied(gbm_ctx *ctx, gbm_ctx::Slot &s) {
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 4, t0, t1));
        TRY(record_ev(ctx, t0, ctx->st));
    }
    TRY(wait_ev(ctx, ctx->st, s.copied));
    if (t1) TRY(record_ev(ctx, t1, ctx->st));
    return GBM_OK;
}

// Fold a slot's finished timing pairs into the totals (each pair once).
int collect_slot_timing(gbm_ctx *ctx, int si) {
    gbm_ctx::Slot &s = ctx->slot[si];
    for (int k = s.tdone; k < s.tused; k++) {
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, s.tev[(size_t)(2 * k)], s.tev[(size_t)(2 * k + 1)]));
        const char kind = s.tkind[(size_t)k];
        (kind == 0 ? ctx->hist_ms : kind == 1 ? ctx->flush_ms : kind == 2 ? ctx->comm_ms
         : kind == 3 ? ctx->samp_ms : ctx->samp_stall_ms) += ms;
    }
    s.tdone = s.tused;
    return GBM_OK;
}

// A round is about to be enqueued on slot si (outside a capture).
// Ranks holding more rows than this build a round's mask and root row list
// after the previous round's levels rather than during them.
constexpr int64_t kEarlyRootRows = 1 << 22;

// The buffer set of round parity q (see d_maskP).
void use_parity(gbm_ctx *ctx, int q) {
    ctx->d_mask = ctx->d_maskP[q];
    ctx->d_rows = ctx->d_rowsP[q];
    ctx->d_tmp = ctx->d_tmpP[q];
    ctx->d_comp = ctx->d_compP[q];
    ctx->d_total = ctx->d_totalP[q];
    ctx->rows_free = ctx->rows_freeP[q];
}

void begin_round(gbm_ctx *ctx, int si) {
    use_parity(ctx, si & 1);
    ctx->cur_slot = si;
    ctx->slot[si].tused = ctx->slot[si].tdone = 0;
}

// (Re)allocation of a context buffer: one that is already big enough is
// kept (a repeated upload of the same shape allocates nothing: cudaFree
// synchronises the device and pinned allocations take milliseconds).  The
// contents are not kept meaningful either way.  mem_gen counts pointer
// changes (captured graphs hold pointers).
template <typename T>
int dalloc(gbm_ctx *ctx, T **p, size_t count) {
    if (count == 0) count = 1;
    const size_t bytes = count * sizeof(T);
    if (*p) {
        auto it = ctx->dcap.find((void *)*p);
        if (it != ctx->dcap.end() && it->second >= bytes) return GBM_OK;
        if (it != ctx->dcap.end()) ctx->dcap.erase(it);
        cudaFree(*p);
        *p = nullptr;
    }
    ctx->mem_gen++;
    cudaError_t e = cudaMalloc((void **)p, bytes);
    if (e != cudaSuccess)
        return fail(ctx, GBM_ERR_ALLOC, "cudaMalloc(%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
    ctx->dcap[(void *)*p] = bytes;
    return GBM_OK;
}

// Frees a buffer dalloc made outside the context's members (a temporary).
template <typename T>
void dfree(gbm_ctx *ctx, T *p) {
    if (!p) return;
    ctx->dcap.erase((void *)p);
    cudaFree(p);
}

template <typename T>
int halloc(gbm_ctx *ctx, T **p, size_t count) {
    if (count == 0) count = 1;
    const size_t bytes = count * sizeof(T);
    if (*p) {
        auto it = ctx->hcap.find((void *)*p);
        if (it != ctx->hcap.end() && it->second >= bytes) return GBM_OK;
        if (it != ctx->hcap.end()) ctx->hcap.erase(it);
        cudaFreeHost(*p);
        *p = nullptr;
    }
    ctx->mem_gen++;
    cudaError_t e = cudaMallocHost((void **)p, bytes);
    if (e != cudaSuccess)
        return fail(ctx, GBM_ERR_ALLOC, "cudaMallocHost(%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
    ctx->hcap[(void *)*p] = bytes;
    return GBM_OK;
}

// ---- predict ---------------------------------------------------------------

// A packed ensemble (_pack_tree_list's arrays, E:2192-2216) -> 8-byte nodes
// and values, with every check that keeps the device walk inside its tree:
// offsets start at 0 and increase (no empty tree), trees hold at most 32767
// nodes, an internal node's feature is below n_features, its threshold is
// not negative (above 255 it is stored as 255 with nanr bit 1: every bin,
// 256 included, goes left, as the reference's compare does), and its
// children lie after it inside its tree, so every walk ends.  Nothing is
// uploaded when a check fails.
int pack_model(std::string &err, const gbm_packed *m, int32_t n_features, std::vector<PNode> &nodes,
               std::vector<double> &vals, std::vector<uint32_t> *n32 = nullptr, std::vector<double> *v32 = nullptr,
               std::vector<int32_t> *dep32 = nullptr, bool *has_nr = nullptr) {
    bool nr_scratch = false;
    if (!has_nr) has_nr = &nr_scratch;
    *has_nr = false;
    auto bad = [&err](int code, const char *fmt, auto... a) {
        char buf[256];
        snprintf(buf, sizeof buf, fmt, a...);
        err = buf;
        return code;
    };
    const int32_t T = m->n_trees;
    if (m->offsets[0] != 0) return bad(GBM_ERR_ARG, "model offsets start at %d, not 0", m->offsets[0]);
    for (int32_t t = 0; t < T; t++) {
        const int32_t o = m->offsets[t], o1 = m->offsets[t + 1];
        if (o1 <= o) return bad(GBM_ERR_ARG, "tree %d is empty or its offsets decrease (%d -> %d)", t, o, o1);
        if (o1 - o > 32767) return bad(GBM_ERR_UNSUPPORTED, "tree %d has %d nodes (at most 32767)", t, o1 - o);
    }
    const int64_t total = m->offsets[T];
    if (total > 0 && (!m->features || !m->thresholds || !m->values || !m->left || !m->right))
        return bad(GBM_ERR_ARG, "%s", "model arrays missing");
    nodes.assign((size_t)std::max<int64_t>(total, 1), PNode{-1, 0, 0, 0, 0});   // feat, thr, nanr, left, right
    vals.assign((size_t)std::max<int64_t>(total, 1), 0.0);
    for (int32_t t = 0; t < T; t++) {
        const int32_t o = m->offsets[t], o1 = m->offsets[t + 1], sz = o1 - o;
        for (int32_t k = o; k < o1; k++) {
            PNode nd{-1, 0, 0, 0, 0};
            const int f = m->features[k];
            if (f >= 0) {
                const int64_t th = m->thresholds[k];
                const int32_t l = m->left[k], r = m->right[k], kk = k - o;
                if (f >= n_features) return bad(GBM_ERR_ARG, "tree %d node %d: feature %d >= %d", t, kk, f, n_features);
                if (th < 0) return bad(GBM_ERR_UNSUPPORTED, "tree %d node %d: negative threshold", t, kk);
                const int nr = m->nan_right && m->nan_right[k] ? 1 : 0;
                if (nr && th < 1)
                    return bad(GBM_ERR_ARG, "tree %d node %d: a NaN-right split needs threshold >= 1", t, kk);
                if (l <= kk || l >= sz || r <= kk || r >= sz)
                    return bad(GBM_ERR_ARG, "tree %d node %d: children %d/%d must lie after the node inside the "
                                "tree (%d nodes)", t, kk, l, r, sz);
                nd.feat = (int16_t)f;
                nd.thr = (uint8_t)(th > 255 ? 255 : th);
                nd.nanr = (uint8_t)(nr | (th > 255 ? 2 : 0));
                nd.left = (int16_t)l;
                nd.right = (int16_t)r;
            }
            nodes[(size_t)k] = nd;
            vals[(size_t)k] = m->values[k];
        }
    }
    if (n32 && v32 && dep32) {
        // the 32-bit breadth-first form (k_predict's PACKED format, the word
        // layout of walk_packed): every tree renumbered so that a node's
        // children are adjacent, each leaf pointing at itself with threshold
        // 255, a NaN-right split stored with threshold - 1 and bit 23 set,
        // and the tree's depth; only when features fit 11 bits and every tree
        // (as reached from its root) fits 4096 nodes, else *n32 stays empty
        n32->clear();
        v32->clear();
        dep32->clear();
        if (n_features > 2048) return GBM_OK;
        std::vector<uint32_t> a((size_t)std::max<int64_t>(total, 1), 0u);
        std::vector<double> b((size_t)std::max<int64_t>(total, 1), 0.0);
        std::vector<int32_t> d((size_t)std::max<int32_t>(T, 1), 0);
        std::vector<int32_t> order, nid, lev;
        for (int32_t t = 0; t < T; t++) {
            const int32_t o = m->offsets[t], sz = m->offsets[t + 1] - o;
            if (sz > 4096) return GBM_OK;
            order.assign(1, 0);
            nid.assign(1, 0);     // nid[i]: the new id of order[i]; lev[i]: its depth
            lev.assign(1, 0);
            int32_t next = 1, depth = 0;
            for (size_t h = 0; h < order.size(); h++) {
                const int32_t k = order[h];
                const PNode &nd = nodes[(size_t)(o + k)];
                uint32_t w = (255u << 24) | (uint32_t)nid[h];   // a leaf: no bin is above 255
                if (nd.feat >= 0) {
                    if (next + 1 >= sz) return GBM_OK;   // more nodes than the tree holds (shared children)
                    // threshold 255 exactly: bin 256 of a 257-bin feature goes right,
                    // which needs the top bits of the 8-byte walk
                    if (nd.thr == 255 && !(nd.nanr & 2)) return GBM_OK;
                    const uint32_t nr = nd.nanr & 1, f = (uint32_t)nd.feat;
                    w = ((uint32_t)(nr ? nd.thr - 1 : nd.thr) << 24) | (nr << 23) | ((f & 3u) << 21) |
                        ((f >> 2) << 12) | (uint32_t)next;
                    if (nr) *has_nr = true;
                    order.push_back(nd.left);
                    nid.push_back(next);
                    lev.push_back(lev[h] + 1);
                    order.push_back(nd.right);
                    nid.push_back(next + 1);
                    lev.push_back(lev[h] + 1);
                    next += 2;
                    depth = std::max(depth, lev[h] + 1);
                }
                a[(size_t)(o + nid[h])] = w;
                b[(size_t)(o + nid[h])] = vals[(size_t)(o + k)];
            }
            d[(size_t)t] = depth;
        }
        n32->swap(a);
        v32->swap(b);
        dep32->swap(d);
    }
    return GBM_OK;
}

// k_predict's shape for p features (kPredThreads threads per CTA, one CTA
// per SM or more when they fit): two rows per thread while that row tile
// fits beside the two chunk buffers; else one row per thread, and fewer
// rows per CTA when even that does not fit; rows wider than 32 rows' tile
// are read from global memory.
struct PredShape {
    int rpt, rpc, stage_rows;
    size_t smem;
};

PredShape predict_shape(int p, bool packed) {
    constexpr size_t kSmem = 227 * 1024;
    if (predict_smem(2 * kPredThreads, p, packed) <= kSmem)
        return {2, 2 * kPredThreads, 1, predict_smem(2 * kPredThreads, p, packed)};
    const size_t room = kSmem - predict_smem(0, p, packed);
    const size_t per32 = predict_smem(32, p, packed) - predict_smem(0, p, packed);
    const int rpc = (int)std::min<size_t>(kPredThreads, room / per32 * 32);
    if (rpc < 32) return {1, kPredThreads, 0, predict_smem(0, p, packed)};   // rows read from global memory
    return {1, rpc, 1, predict_smem(rpc, p, packed)};
}

template <int RPT, bool PK, bool SR, bool NR>
cudaError_t launch_predict_t(const PredShape &sh, unsigned grid, const uint8_t *xr, int64_t n, int p,
                             const void *nodes, const double *vals, const int32_t *off, const int32_t *dep, int ntree,
                             const int4 *cstart, const int32_t *nchunk, double lr, double base, double *F,
                             double *P, const int32_t *bigidx, const uint32_t *topbits, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(k_predict<RPT, PK, SR, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sh.smem);
    if (e != cudaSuccess) return e;
    k_predict<RPT, PK, SR, NR><<<grid, kPredThreads, sh.smem, st>>>(xr, n, p, nodes, vals, off, dep, ntree, cstart,
                                                                 nchunk, sh.rpc, lr, base, F, P, bigidx,
                                                                 topbits);
    return cudaGetLastError();
}

// The ensemble over n rows (row-major bins [n][p]); chunk starts and count
// were written by k_pred_chunks.  `packed`: nodes are 32-bit breadth-first
// words with per-tree depths `dep` (pack_model), else PNode (dep unused).
// bigidx [p] / topbits [big][ceil(n / 32)]: the rows of bin 256 of 257-bin
// features (null: none; only the PNode walk reads them).  Allocates nothing.
cudaError_t launch_predict(const uint8_t *xr, int64_t n, int p, const void *nodes, bool packed, const double *vals,
                           const int32_t *off, const int32_t *dep, int ntree, const int4 *cstart,
                           const int32_t *nchunk, double lr, double base, double *F, double *P,
                           const int32_t *bigidx, const uint32_t *topbits, cudaStream_t st, bool packed_nr = true) {
    PredShape sh = predict_shape(p, packed);
    if (sh.stage_rows && n > 0) {
        // whole waves: the fewest waves of full SMs at the shape's rows per
        // CTA, then the rows spread evenly over them (a multiple of 32 rows
        // per CTA, at most the shape's)
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int per_sm = std::max<int>(1, std::min<int>(2048 / kPredThreads, (int)((228 * 1024) / (sh.smem + 1024))));
        const int64_t slots = (int64_t)std::max(1, sms) * per_sm;
        const int64_t waves = (n + slots * sh.rpc - 1) / (slots * sh.rpc);
        const int64_t even = ((n + waves * slots - 1) / (waves * slots) + 31) / 32 * 32;
        if (even < sh.rpc) {
            sh.rpc = (int)std::max<int64_t>(32, even);
            sh.smem = predict_smem(sh.rpc, p, packed);
        }
    }
    const unsigned grid = (unsigned)((n + sh.rpc - 1) / sh.rpc);
#define GBM_PRED(R, K, S, N) launch_predict_t<R, K, S, N>(sh, grid, xr, n, p, nodes, vals, off, dep, ntree, cstart, nchunk, lr, base, F, P, bigidx, topbits, st)
    if (packed) {   // NaN-right splits in the packed words: the walk's extra step only when the model has some
        if (sh.rpt == 2) return packed_nr ? GBM_PRED(2, true, true, true) : GBM_PRED(2, true, true, false);
        if (sh.stage_rows) return packed_nr ? GBM_PRED(1, true, true, true) : GBM_PRED(1, true, true, false);
        return packed_nr ? GBM_PRED(1, true, false, true) : GBM_PRED(1, true, false, false);
    }
    if (sh.rpt == 2) return GBM_PRED(2, false, true, false);
    if (sh.stage_rows) return GBM_PRED(1, false, true, false);
    return GBM_PRED(1, false, false, false);
#undef GBM_PRED
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

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

int sync_stream(gbm_ctx *ctx) {
    auto t0 = std::chrono::steady_clock::now();
    int rc = GBM_OK;
    if (ctx->comm) {
        rc = gbm_comm_sync(ctx->comm, ctx->st, ctx->timeout_ms, ctx->err);
    } else {
        cudaError_t e = cudaStreamSynchronize(ctx->st);
        if (e != cudaSuccess) rc = fail(ctx, GBM_ERR_CUDA, "stream sync: %s", cudaGetErrorString(e));
    }
    ctx->host_sync_ms += ms_since(t0);
    return rc;
}

// In-place sums over the ranks on the engine stream; host time counted, and
// device time (waiting for the peers included) when profiling.
int allreduce_i64(gbm_ctx *ctx, long long *buf, int64_t count) {
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 2, e0, e1));
        TRY(record_ev(ctx, e0, ctx->st));
    }
    auto t0 = std::chrono::steady_clock::now();
    int rc = gbm_comm_allreduce_i64(ctx->comm, buf, count, ctx->st, ctx->timeout_ms, ctx->err);
    ctx->host_comm_ms += ms_since(t0);
    if (rc == GBM_OK && e1) TRY(record_ev(ctx, e1, ctx->st));
    ctx->comm_bytes += 8.0 * (double)count;
    return rc;
}

int allreduce_f64(gbm_ctx *ctx, double *buf, int64_t count) {
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 2, e0, e1));
        TRY(record_ev(ctx, e0, ctx->st));
    }
    auto t0 = std::chrono::steady_clock::now();
    int rc = gbm_comm_allreduce_f64(ctx->comm, buf, count, ctx->st, ctx->timeout_ms, ctx->err);
    ctx->host_comm_ms += ms_since(t0);
    if (rc == GBM_OK && e1) TRY(record_ev(ctx, e1, ctx->st));
    ctx->comm_bytes += 8.0 * (double)count;
    return rc;
}

// ---- per-round feature tables ---------------------------------------------

struct RoundFeat {
    int nf;
    std::vector<int32_t> blist;
    std::vector<int16_t> fpos;
    double upd_per_row = 0.0;   // histogram cell updates per row: the selected features
};

// The histograms read the round's packed feature blocks (k_compact_feat):
// the default (GBM_HIST_COMPACT unset or 1) whenever the compaction's staging
// of 256 rows x every column block fits its shared memory (p <= 608).
bool compact_hist(const gbm_ctx *ctx) {
    return ctx->hist_compact && ctx->nblk <= 38;
}

// Per-slot pinned staging, sized for the data.
int ensure_slots(gbm_ctx *ctx) {
    if (!ctx->slots_ready) {   // once per gbm_upload_bins (sizes follow p)
        for (auto &s : ctx->slot) {
            TRY(halloc(ctx, &s.h_feat, (size_t)ctx->p + 2 * ctx->nblk + 2));
            TRY(dalloc(ctx, &s.d_fidx_c, (size_t)ctx->p));
            TRY(halloc(ctx, &s.h_round, 1));
            TRY(dalloc(ctx, &s.d_round, 1));
            TRY(halloc(ctx, &s.h_fpos, (size_t)ctx->nblk * kBlk + ctx->p));
            TRY(halloc(ctx, &s.h_tout, 1));
            TRY(halloc(ctx, &s.h_loss, 2));   // [0] loss, [1] the peer exchange's error word
            if (!s.copied) CK(cudaEventCreateWithFlags(&s.copied, cudaEventDisableTiming));
            if (!s.done) CK(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
        }
        TRY(dalloc(ctx, &ctx->d_tout, 1));
        TRY(dalloc(ctx, &ctx->d_mono, (size_t)ctx->p));
        TRY(dalloc(ctx, &ctx->d_nanf, (size_t)ctx->p));
        TRY(halloc(ctx, &ctx->h_nanf, (size_t)ctx->p));
        TRY(halloc(ctx, &ctx->h_mono, (size_t)ctx->p));
        ctx->slots_ready = true;
    }
    return GBM_OK;
}

// Row shuffle buffers for a sampler over N global rows.
int ensure_shuffle(gbm_ctx *ctx, int64_t N) {
    if (N <= ctx->shuf_n) return GBM_OK;
    for (auto &s : ctx->slot) {
        TRY(halloc(ctx, &s.h_tg, (size_t)N + 8));
        TRY(dalloc(ctx, &s.d_tg, (size_t)N + 8));
    }
    for (auto &q : ctx->d_perm) TRY(dalloc(ctx, &q, (size_t)N));
    TRY(dalloc(ctx, &ctx->d_head, (size_t)N));
    TRY(dalloc(ctx, &ctx->d_nxt, (size_t)N));
    TRY(dalloc(ctx, &ctx->d_m, (size_t)N));
    TRY(dalloc(ctx, &ctx->d_mp, (size_t)N));
    ctx->shuf_n = N;
    return GBM_OK;
}

// The round's feature tables, built in the slot's pinned buffers (host).
int setup_features(gbm_ctx *ctx, int si, const int32_t *fidx, int nf, RoundFeat &rf) {
    gbm_ctx::Slot &s = ctx->slot[si];
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
    const int nb = (int)rf.blist.size();
    int32_t *h_blist = s.h_feat + ctx->p;
    int16_t *h_fbi = s.h_fpos + (size_t)ctx->nblk * kBlk;
    std::memcpy(s.h_feat, fidx, sizeof(int32_t) * nf);
    std::memcpy(h_blist, rf.blist.data(), sizeof(int32_t) * nb);
    for (int bi = 0; bi < nb; bi++) {
        for (int k = 0; k < kBlk; k++) {
            int jj = rf.fpos[(size_t)rf.blist[bi] * kBlk + k];
            if (jj >= 0) h_fbi[jj] = (int16_t)bi;
        }
    }
    h_blist[ctx->nblk] = nb;   // the count, after the longest list
    std::memcpy(s.h_fpos, rf.fpos.data(), sizeof(int16_t) * rf.fpos.size());
    rf.upd_per_row = nf;
    s.upd_per_row = rf.upd_per_row;
    return GBM_OK;
}

// The round's selected features packed into blocks of 16 (k_compact_feat),
// on stream st.
int enqueue_pack(gbm_ctx *ctx, cudaStream_t st, const int32_t *d_fidx, int nf, uint8_t *xc) {
    const size_t smem = (size_t)ctx->nblk * kCompactRows * kCompactStrideW * 4 + sizeof(int32_t) * (size_t)nf;
    return launch(ctx, k_compact_feat, dim3((unsigned)((ctx->n + kCompactRows - 1) / kCompactRows)),
                  dim3(kCompactRows), smem, st, (const uint8_t *)ctx->d_xb, ctx->n, ctx->nblk, d_fidx, nf, xc);
}

// ...and their copies to the device, on the engine stream (fixed sizes, so
// a captured round copies whatever the slot holds when it runs).
int enqueue_features(gbm_ctx *ctx, int si, int nf) {
    gbm_ctx::Slot &s = ctx->slot[si];
    CK(cudaMemcpyAsync(ctx->d_fidx, s.h_feat, sizeof(int32_t) * nf, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_fpos, s.h_fpos, sizeof(int16_t) * (size_t)ctx->nblk * kBlk, cudaMemcpyHostToDevice,
                       ctx->st));
    CK(cudaMemcpyAsync(ctx->d_fbi, s.h_fpos + (size_t)ctx->nblk * kBlk, sizeof(int16_t) * nf, cudaMemcpyHostToDevice,
                       ctx->st));
    CK(cudaMemcpyAsync(ctx->d_blist, s.h_feat + ctx->p, sizeof(int32_t) * ((size_t)ctx->nblk + 1),
                       cudaMemcpyHostToDevice, ctx->st));
    const bool packed_on_cst = s.xc_on_cst;
    s.xc_on_cst = false;   // a later round in this slot may take another path
    if (compact_hist(ctx)) {   // the round's selected features, packed for the histograms
        if (packed_on_cst) {
            ctx->xc_cur = ctx->d_xc[si & 1];   // packed on cst before s.copied
        } else {
            TRY(enqueue_pack(ctx, ctx->st, ctx->d_fidx, nf, ctx->d_xc[0]));
            ctx->xc_cur = ctx->d_xc[0];
        }
    }
    return GBM_OK;
}

// Level widths: level L expands at most min(2^L, M) parents.  Depth-wise
// growth and best-first growth up to depth kSpecDepth use M = 2^(D-1), so
// every node that can split is expanded and the tree is replayed on the
// device with no host round trip.  Deeper best-first trees use M =
// max_leaves - 1 (no tree uses more splits) and expand on demand what the
// ranking left out.
constexpr int kSpecDepth = 10;
constexpr int kReplaySmemMax = 160 * 1024;   // node table copy of the replay kernels

// The deepest best-first tree grown with full speculation: kSpecDepth, or
// lower with GBM_SPEC_DEPTH in the environment (0: every best-first tree
// takes capped speculation and the host replay).
int spec_depth() {
    static const int d = [] {
        const char *e = std::getenv("GBM_SPEC_DEPTH");
        return e ? std::max(0, std::min(kSpecDepth, std::atoi(e))) : kSpecDepth;
    }();
    return d;
}

bool full_spec(const gbm_params *P) { return P->grow_policy == 1 || P->max_depth <= spec_depth(); }

// Children below this depth keep their histogram in the pool (a future
// parent's).  Under full speculation the nodes at depth D-1 are expanded by
// the last level, which needs no histogram; otherwise any node may still be
// expanded on demand.
int pool_depth(const gbm_params *P) { return full_spec(P) ? P->max_depth - 1 : 1 << 30; }

// Best-first trees grown with full speculation skip the nodes the
// reference's loop can never split (k_level_close) when the depth allows
// many more splits than max_leaves - 1 (a depth-6, 63-leaf tree has nothing
// to skip); GBM_PRUNE=0 keeps every node.
bool prune_best_first(const gbm_params *P) {
    static const bool on = [] {
        const char *e = std::getenv("GBM_PRUNE");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    const long long splits = P->max_depth >= 40 ? (1ll << 40) : (1ll << P->max_depth) - 1;
    return on && P->grow_policy == 0 && full_spec(P) && splits > 2ll * (P->max_leaves - 1);
}

int level_cap(const gbm_params *P) {
    if (P->grow_policy == 1) return 1 << std::min(P->max_depth - 1, 12);
    int m = std::max(1, P->max_leaves - 1);
    if (full_spec(P)) m = std::max(m, 1 << (P->max_depth - 1));
    return m;
}

int level_width(const gbm_params *P, int L) {
    int w = L >= 20 ? (1 << 20) : (1 << L);
    return std::min(w, level_cap(P));
}

// ---- peer exchange setup (several ranks) -----------------------------------------

// Unmaps the peers' buffers and frees this rank's.  `collective`: the ranks
// first agree (an all-reduce) that nobody reads them any more.
int p2p_teardown(gbm_ctx *ctx, bool collective) {
    if (!ctx->d_pst && !ctx->d_sync && ctx->ipc_opened.empty()) return GBM_OK;
    if (ctx->st) cudaStreamSynchronize(ctx->st);
    if (collective && ctx->comm) {
        TRY(allreduce_i64(ctx, ctx->d_count64, 1));
        TRY(sync_stream(ctx));
    }
    for (void *q : ctx->ipc_opened) cudaIpcCloseMemHandle(q);
    ctx->ipc_opened.clear();
    if (collective && ctx->comm) {   // every rank has unmapped this rank's buffers
        TRY(allreduce_i64(ctx, ctx->d_count64, 1));
        TRY(sync_stream(ctx));
    }
    void *ptrs[] = {ctx->d_pst, ctx->d_sync, ctx->d_red, ctx->d_peer_pst, ctx->d_peer_sync, ctx->d_peer_red};
    for (void *q : ptrs) if (q) cudaFree(q);
    ctx->d_pst = nullptr;
    ctx->d_sync = nullptr;
    ctx->d_red = nullptr;
    ctx->d_peer_pst = nullptr;
    ctx->d_peer_sync = nullptr;
    ctx->d_peer_red = nullptr;
    ctx->pst_stride = 0;
    ctx->p2p = false;
    ctx->mem_gen++;
    return GBM_OK;
}

// Collective: every rank calls it at the same point.  Allocates the two
// parity staging buffers and the sync words, exchanges their CUDA IPC
// handles through the communicator (an all-reduce of a zeroed table into
// which each rank writes its own row) and maps every peer's.  If any rank
// cannot export or map, all ranks stay on the NCCL all-reduce.
// GBM_PEER_EXCHANGE=0 turns the exchange off.
int p2p_setup(gbm_ctx *ctx, int64_t stride) {
    TRY(p2p_teardown(ctx, true));
    const char *env = std::getenv("GBM_PEER_EXCHANGE");
    const int N = gbm_comm_size(ctx->comm), rank = gbm_comm_rank(ctx->comm);
    // default on for 2 ranks, where it beats the NCCL all-reduce (983 vs 946 rounds/s for config 4);
    // at 4 ranks NCCL's all-reduce is the faster (967 vs 858 for the two-shot exchange).
    // GBM_PEER_EXCHANGE=1 turns it on for any count, 0 off.
    if (env ? env[0] == '0' : N != 2) return GBM_OK;
    ctx->p2p_n = N;
    ctx->p2p_rank = rank;
    int ok = 1;
    const size_t sync_words = (size_t)(2 * N + kSyncLocal);
    if (cudaMalloc(&ctx->d_pst, sizeof(long long) * (size_t)(2 * stride)) != cudaSuccess ||
        cudaMalloc(&ctx->d_red, sizeof(long long) * (size_t)stride) != cudaSuccess ||
        cudaMalloc(&ctx->d_sync, sizeof(unsigned long long) * sync_words) != cudaSuccess ||
        cudaMalloc(&ctx->d_peer_pst, sizeof(long long *) * (size_t)N) != cudaSuccess ||
        cudaMalloc(&ctx->d_peer_red, sizeof(long long *) * (size_t)N) != cudaSuccess ||
        cudaMalloc(&ctx->d_peer_sync, sizeof(unsigned long long *) * (size_t)N) != cudaSuccess)
        return fail(ctx, GBM_ERR_ALLOC, "peer exchange buffers");
    ctx->mem_gen++;
    CK(cudaMemsetAsync(ctx->d_pst, 0, sizeof(long long) * (size_t)(2 * stride), ctx->st));
    CK(cudaMemsetAsync(ctx->d_sync, 0, sizeof(unsigned long long) * sync_words, ctx->st));
    // the handle table: per rank 3 handles of 64 bytes = 24 int64 words
    constexpr int kNH = 3;
    constexpr int kHW = (int)(kNH * sizeof(cudaIpcMemHandle_t) / 8);
    static_assert(kNH * sizeof(cudaIpcMemHandle_t) == 8 * kHW, "handle size");
    std::vector<long long> tab((size_t)N * kHW + 1, 0);
    cudaIpcMemHandle_t h[kNH];
    if (cudaIpcGetMemHandle(&h[0], ctx->d_pst) != cudaSuccess || cudaIpcGetMemHandle(&h[1], ctx->d_sync) != cudaSuccess ||
        cudaIpcGetMemHandle(&h[2], ctx->d_red) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
    } else {
        std::memcpy(&tab[(size_t)rank * kHW], h, sizeof h);
    }
    tab[(size_t)N * kHW] = ok ? 0 : 1;   // ranks that failed
    long long *d_tab = nullptr;
    TRY(dalloc(ctx, &d_tab, tab.size()));
    CK(cudaMemcpyAsync(d_tab, tab.data(), sizeof(long long) * tab.size(), cudaMemcpyHostToDevice, ctx->st));
    int rc = allreduce_i64(ctx, d_tab, (int64_t)tab.size());
    if (rc == GBM_OK) rc = cudaMemcpyAsync(tab.data(), d_tab, sizeof(long long) * tab.size(), cudaMemcpyDeviceToHost,
                                           ctx->st) == cudaSuccess ? sync_stream(ctx) : GBM_ERR_CUDA;
    dfree(ctx, d_tab);
    if (rc != GBM_OK) return rc;
    std::vector<long long *> pst((size_t)N, nullptr), red((size_t)N, nullptr);
    std::vector<unsigned long long *> sy((size_t)N, nullptr);
    pst[(size_t)rank] = ctx->d_pst;
    sy[(size_t)rank] = ctx->d_sync;
    red[(size_t)rank] = ctx->d_red;
    if (tab[(size_t)N * kHW] == 0) {
        for (int q = 0; q < N && ok; q++) {
            if (q == rank) continue;
            cudaIpcMemHandle_t hq[kNH];
            std::memcpy(hq, &tab[(size_t)q * kHW], sizeof hq);
            void *m[kNH] = {};
            for (int k = 0; k < kNH && ok; k++) {
                if (cudaIpcOpenMemHandle(&m[k], hq[k], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                    cudaGetLastError();
                    ok = 0;
                    break;
                }
                ctx->ipc_opened.push_back(m[k]);
            }
            pst[(size_t)q] = static_cast<long long *>(m[0]);
            sy[(size_t)q] = static_cast<unsigned long long *>(m[1]);
            red[(size_t)q] = static_cast<long long *>(m[2]);
        }
    }
    // every rank must map every peer, or nobody uses the exchange
    CK(cudaMemsetAsync(ctx->d_count64, 0, sizeof(long long), ctx->st));
    if (!ok) {
        long long one = 1;
        CK(cudaMemcpyAsync(ctx->d_count64, &one, sizeof one, cudaMemcpyHostToDevice, ctx->st));
    }
    TRY(allreduce_i64(ctx, ctx->d_count64, 1));
    long long bad = 0;
    CK(cudaMemcpyAsync(&bad, ctx->d_count64, sizeof bad, cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    if (bad || tab[(size_t)N * kHW]) return p2p_teardown(ctx, true);
    CK(cudaMemcpyAsync(ctx->d_peer_pst, pst.data(), sizeof(long long *) * (size_t)N, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_peer_sync, sy.data(), sizeof(unsigned long long *) * (size_t)N, cudaMemcpyHostToDevice,
                       ctx->st));
    CK(cudaMemcpyAsync(ctx->d_peer_red, red.data(), sizeof(long long *) * (size_t)N, cudaMemcpyHostToDevice, ctx->st));
    TRY(sync_stream(ctx));
    ctx->pst_stride = stride;
    ctx->p2p = true;
    return GBM_OK;
}

// A round's exchange ran out of time on this rank (the flag copied into the
// slot's pinned words with the round).
int p2p_check(gbm_ctx *ctx, int si) {
    if (!ctx->p2p) return GBM_OK;
    unsigned long long e = 0;
    std::memcpy(&e, &ctx->slot[si].h_loss[1], sizeof e);
    if (e) return fail(ctx, GBM_ERR_TIMEOUT, "peer exchange: a peer did not reach a level in time (a rank may have left)");
    return GBM_OK;
}

int ensure_round_buffers(gbm_ctx *ctx, int nf, const gbm_params *P) {
    int need_nf = std::max(nf, 1);
    int stage = std::max(level_cap(P), P->grow_policy == 0 ? P->max_leaves + 2 : 1);
    int nodes = 1;
    for (int L = 0; L < P->max_depth; L++) nodes += 2 * level_width(P, L);
    nodes += 2 * (P->max_leaves + 2) + 8;   // on-demand expansions during the replay
    if (need_nf > ctx->nf_cap || stage > ctx->stage_slots || nodes > ctx->nmax) {
        ctx->nf_cap = std::max(need_nf, ctx->nf_cap);
        ctx->stage_slots = std::max(stage, ctx->stage_slots);
        ctx->nmax = std::max(nodes, ctx->nmax);
        int64_t words = slot_words_for(ctx->nf_cap);
        TRY(dalloc(ctx, &ctx->d_pool, (size_t)ctx->nmax * words));
        TRY(dalloc(ctx, &ctx->d_stage, (size_t)ctx->stage_slots * words));
        TRY(dalloc(ctx, &ctx->d_fidx, (size_t)ctx->nf_cap));
        TRY(dalloc(ctx, &ctx->d_fbest, (size_t)2 * ctx->stage_slots * ctx->nf_cap));
        TRY(dalloc(ctx, &ctx->d_nodes, (size_t)ctx->nmax));
        TRY(halloc(ctx, &ctx->h_nodes, (size_t)ctx->nmax));
        TRY(dalloc(ctx, &ctx->d_lvl[0], (size_t)ctx->stage_slots + 1));
        TRY(dalloc(ctx, &ctx->d_lvl[1], (size_t)ctx->stage_slots + 1));
        TRY(halloc(ctx, &ctx->h_list, (size_t)ctx->stage_slots + 1));
        TRY(dalloc(ctx, &ctx->d_htask, (size_t)ctx->stage_slots));
        TRY(dalloc(ctx, &ctx->d_hprefix, (size_t)ctx->stage_slots + 1));
        TRY(dalloc(ctx, &ctx->d_ptask, (size_t)ctx->stage_slots));
        TRY(dalloc(ctx, &ctx->d_nleft, (size_t)ctx->stage_slots));
        TRY(dalloc(ctx, &ctx->d_leafw, (size_t)ctx->stage_slots * kLeafWords));
        int smem = (int)(sizeof(RNode) * (size_t)ctx->nmax);
        ctx->replay_smem = 0;
        if (smem <= kReplaySmemMax) ctx->replay_smem = smem;
    }
    if (ctx->comm) {
        const int64_t lw = (int64_t)ctx->nmax * slot_words_for(ctx->nf_cap);
        if (lw > ctx->lpool_words) {
            TRY(dalloc(ctx, &ctx->d_lpool, (size_t)lw));
            ctx->lpool_words = lw;
        }
        const int64_t stride = (int64_t)ctx->stage_slots * slot_words_for(ctx->nf_cap);
        if (stride != ctx->p2p_tried_stride) {
            ctx->p2p_tried_stride = stride;
            TRY(p2p_setup(ctx, stride));
        }
    }
    const int tiles = (int)((ctx->n + kPartTile - 1) / kPartTile) + ctx->stage_slots;
    if (tiles > ctx->tile_cap) {
        ctx->tile_cap = tiles;
        TRY(dalloc(ctx, &ctx->d_tile_st, (size_t)ctx->tile_cap));
        CK(cudaMemsetAsync(ctx->d_tile_st, 0, sizeof(unsigned long long) * ctx->tile_cap, ctx->st));
    }
    return GBM_OK;
}

// The tree can be replayed on the device: every node it can need is
// expanded, and the node table fits the replay's shared-memory copy.
bool device_replay(const gbm_ctx *ctx, const gbm_params *P) {
    return full_spec(P) && ctx->replay_smem > 0 && ctx->replay_smem >= (int)(sizeof(RNode) * (size_t)ctx->nmax);
}

// ---- launches -----------------------------------------------------------------

// The histograms of the tasks at *ntask_p: one k_hist3 CTA per SM.
// The staging histograms are zero here: the split search zeroes the cells
// it reads and the level close the totals.
int launch_hist(gbm_ctx *ctx, const RoundFeat &rf, const int *ntask_p) {
    // d_blist holds blist [nblk] | nb
    const int32_t *d_nb = ctx->d_blist + ctx->nblk;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 0, e0, e1));
        TRY(record_ev(ctx, e0, ctx->st));
    }
    long long *stage = ctx->p2p ? ctx->d_pst : ctx->d_stage;
    const unsigned long long *par = (const unsigned long long *)(ctx->p2p ? ctx->d_sync + ctx->p2p_n + kSyncLevel
                                                                          : nullptr);
    const size_t hsm = (size_t)kAccV3Words * sizeof(unsigned);
    const uint8_t *hx = compact_hist(ctx) ? ctx->xc_cur : ctx->d_xb;
#define GBM_HIST3(C)                                                                                          \
    launch(ctx, k_hist3<C>, dim3(ctx->sms), dim3(kHistV3Threads), hsm, ctx->st, hx, ctx->n, ctx->d_rows,      \
           ctx->d_tmp, ctx->d_htask, ctx->d_hprefix, ntask_p, ctx->d_blist, d_nb, ctx->d_fpos, rf.nf, ctx->d_q, \
           stage, par, ctx->pst_stride, ctx->hist_seg_cost)
    if (compact_hist(ctx)) TRY(GBM_HIST3(true));
    else TRY(GBM_HIST3(false));
#undef GBM_HIST3
    if (ctx->nbig)   // bin 256 of the 257-bin features, into the top cells
        TRY(launch(ctx, k_hist_top, dim3(ctx->nbig), dim3(128), 0, ctx->st, (const int32_t *)ctx->d_rows,
                   (const int32_t *)ctx->d_tmp, (const HistTask *)ctx->d_htask, ntask_p,
                   (const int32_t *)ctx->d_bigfeat, (const int16_t *)ctx->d_fpos, (const int32_t *)ctx->d_topoff,
                   (const int32_t *)ctx->d_toprows, rf.nf, (const longlong2 *)ctx->d_q, stage, par,
                   ctx->pst_stride));
    if (e1) TRY(record_ev(ctx, e1, ctx->st));
    ctx->hist_launches++;
    return GBM_OK;
}


// The L2 eviction of gbm_set_l2_flush: a write of the scratch buffer on the
// engine stream before the round's growth (timed when profiling).
int flush_l2(gbm_ctx *ctx) {
    if (!ctx->flush_bytes) return GBM_OK;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 1, e0, e1));
        TRY(record_ev(ctx, e0, ctx->st));
    }
    CK(cudaMemsetAsync(ctx->d_flush, (int)(++ctx->flush_count & 0xff), ctx->flush_bytes, ctx->st));
    if (e1) TRY(record_ev(ctx, e1, ctx->st));
    return GBM_OK;
}

int *ints(gbm_ctx *ctx, int i) { return ctx->d_ints + i; }

// The next level a level-synchronous close plans: its list capacity, and
// whether it is the last level (children at max_depth).
struct NextPlan {
    int W_ub = 0;       // 0: no plan (the caller plans, or there is no next level)
    bool last = false;
};

int launch_close(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, bool root, const int *lvl,
                 const int *lvl_cnt, int *next, int *next_cnt, const NextPlan &np) {
    PartTask *pt = np.W_ub > 0 ? ctx->d_ptask : nullptr;
    long long *lw = np.W_ub > 0 && np.last ? ctx->d_leafw : nullptr;
    if (root)
        TRY(launch(ctx, k_level_close<true>, dim3(1), dim3(kCloseThreads), 0, ctx->st,
            ctx->d_nodes, nullptr, nullptr, ctx->d_pool, ctx->d_stage, rf.nf, ctx->d_fidx, ctx->d_fbest, ctx->S, next,
            next_cnt, ints(ctx, I_NODES), ctx->nmax, level_cap(P), P->gamma, P->grow_policy == 0, pt,
            ints(ctx, I_TILES), np.W_ub, lw, ctx->d_nleft, 0, (long long)P->min_samples_leaf, P->max_leaves));
    else
        TRY(launch(ctx, k_level_close<false>, dim3(1), dim3(kCloseThreads), 0, ctx->st, 
            ctx->d_nodes, lvl, lvl_cnt, ctx->d_pool, ctx->d_stage, rf.nf, ctx->d_fidx, ctx->d_fbest, ctx->S, next,
            next_cnt, ints(ctx, I_NODES), ctx->nmax, level_cap(P), P->gamma, P->grow_policy == 0, pt,
            ints(ctx, I_TILES), np.W_ub, lw, ctx->d_nleft, prune_best_first(P) ? 1 : 0,
            (long long)P->min_samples_leaf, P->max_leaves));
    return GBM_OK;
}

// Root: histogram of all in-bag rows, its split, the first level list and
// that level's plan.
// The limit of one level's wait for the peers: the communicator's timeout,
// at most GBM_PEER_WAIT_MS (default 10 s; a level takes milliseconds).
long long peer_wait_ns(const gbm_ctx *ctx) {
    long long ms = 10000;
    if (const char *e = std::getenv("GBM_PEER_WAIT_MS")) ms = std::max(1ll, std::atoll(e));
    return std::min<long long>(ms, ctx->timeout_ms) * 1000000ll;
}

// The sum over ranks of the level's staging slots into d_stage: the peer
// exchange (k_peer_sum), or an NCCL all-reduce in place.
int exchange_stage(gbm_ctx *ctx, const int *lvl_cnt, int W_ub, int nf) {
    const int64_t words = slot_words_for(nf);
    if (!ctx->p2p) return allreduce_i64(ctx, ctx->d_stage, words * W_ub);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 2, e0, e1));
        TRY(record_ev(ctx, e0, ctx->st));
    }
    const int64_t n2 = (int64_t)W_ub * words / 2;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n2 + 1023) / 1024, 2 * ctx->hist_grid));
    const int N = ctx->p2p_n;
    if (N == 2) {   // one-shot: pull the whole level from the other rank
        TRY(launch(ctx, k_peer_sum, dim3(grid), dim3(256), 0, ctx->st, (const long long *const *)ctx->d_peer_pst,
                   ctx->pst_stride, ctx->d_sync, ctx->p2p_rank, N, lvl_cnt, nf, ctx->d_stage, ctx->d_pst,
                   peer_wait_ns(ctx)));
        ctx->comm_bytes += 8.0 * (double)(words * W_ub);
    } else {        // two-shot: sum this rank's share from every rank, then gather the shares
        const int g1 = std::max(1, grid / N);
        TRY(launch(ctx, k_peer_reduce, dim3(g1), dim3(256), 0, ctx->st, (const long long *const *)ctx->d_peer_pst,
                   ctx->pst_stride, ctx->d_sync, (unsigned long long *const *)ctx->d_peer_sync, ctx->p2p_rank, N,
                   lvl_cnt, nf, ctx->d_red, peer_wait_ns(ctx)));
        TRY(launch(ctx, k_peer_gather, dim3(grid), dim3(256), 0, ctx->st, (const long long *const *)ctx->d_peer_red,
                   ctx->d_sync, ctx->p2p_rank, N, lvl_cnt, nf, ctx->d_stage, ctx->d_pst, ctx->pst_stride,
                   peer_wait_ns(ctx)));
        ctx->comm_bytes += 8.0 * (double)(words * W_ub) * 2.0 * (N - 1) / N;
    }
    if (e1) TRY(record_ev(ctx, e1, ctx->st));
    return GBM_OK;
}

// Several ranks: one exchange per histogram level.  The root's row count
// travels in its staging slot's count word; each level's left counts in the
// slots' count words (k_stage_left / k_fill_counts), so the partition needs
// no collective of its own.
int launch_root(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, const NextPlan &np) {
    long long *sbase = ctx->p2p ? ctx->d_pst : ctx->d_stage;
    unsigned long long *sync = ctx->p2p ? ctx->d_sync : nullptr;
    const unsigned long long *par = sync ? sync + ctx->p2p_n + kSyncLevel : nullptr;
    long long *cw = ctx->comm ? sbase + (int64_t)rf.nf * kBins * kWords + kCountWord : nullptr;
    TRY(launch(ctx, k_root_plan, dim3(1), dim3(1), 0, ctx->st, ctx->d_total, (const long long *)nullptr, ctx->d_nodes,
               ctx->d_htask, ctx->d_hprefix, ints(ctx, I_NODES), cw, par, ctx->pst_stride));
    TRY(launch_hist(ctx, rf, ints(ctx, I_ONE)));
    if (ctx->comm) {
        // this rank's root partial into lpool[0], for the first level's subtractions
        TRY(launch(ctx, k_stage_left, dim3(std::max(1, 2 * ctx->hist_grid / 8), 1), dim3(256), 0, ctx->st,
                   (const DNode *)ctx->d_nodes, (const int *)nullptr, (const int *)nullptr, ctx->d_htask, sbase,
                   ctx->pst_stride, ctx->d_lpool, rf.nf, pool_depth(P), sync,
                   (unsigned long long *const *)ctx->d_peer_sync, ctx->p2p_rank, ctx->p2p_n));
        TRY(exchange_stage(ctx, nullptr, 1, rf.nf));
        TRY(launch(ctx, k_fill_counts, dim3(1), dim3(32), 0, ctx->st, ctx->d_nodes, (const int *)nullptr,
                   (const int *)nullptr, (const long long *)ctx->d_stage, rf.nf, sync, ctx->p2p_n));
    }
    TRY(launch(ctx, k_split_bins<true>, dim3(rf.nf, 1), dim3(kSplitThreads), 0, ctx->st,
        (const DNode *)ctx->d_nodes, (const int *)nullptr, (const int *)nullptr, (const HistTask *)ctx->d_htask,
        ctx->d_stage, ctx->d_pool, rf.nf, (const int32_t *)ctx->d_fidx, (const int32_t *)ctx->d_counts,
        (const uint8_t *)(ctx->nan_dir ? ctx->d_nanf : nullptr), ctx->S, P->reg_lambda, P->min_child_weight,
        (long long)P->min_samples_leaf, P->max_depth, pool_depth(P), ctx->d_fbest));
    return launch_close(ctx, rf, P, true, nullptr, nullptr, ctx->d_lvl[0], ints(ctx, I_LVL0), np);
}

// Expand the parents in `lvl` (count at *lvl_cnt, at most W_ub): partition,
// smaller-child histogram, subtraction, children's splits.  `planned`: the
// previous close planned this level; otherwise (on-demand expansion) it is
// planned here.  `last`: the children are at max_depth (counts and totals
// only).  When `next` is given, the close ranks the children into the next
// level list and, with np.W_ub > 0, plans that level.
int launch_level(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, int *lvl, int *lvl_cnt,
                 int *next, int *next_cnt, int W_ub, bool last, bool planned, const NextPlan &np, int hist_level) {
    if (W_ub <= 0) return GBM_OK;
    const int64_t words = slot_words_for(rf.nf);
    if (!planned) {
        TRY(launch(ctx, k_lvl_plan, dim3(1), dim3(256), 0, ctx->st, ctx->d_nodes, lvl, lvl_cnt, ints(ctx, I_NODES), ctx->d_ptask,
                                           ints(ctx, I_TILES), ctx->nmax, W_ub));
    }
    int tiles_ub = (int)((ctx->n + kPartTile - 1) / kPartTile) + W_ub;
    if (tiles_ub > ctx->tile_cap)   // ensure_round_buffers sized them
        return fail(ctx, GBM_ERR_STATE, "internal: %d partition tiles > %d", tiles_ub, ctx->tile_cap);
    if (last) {   // children at max_depth: counts and totals only
        if (!planned) {
            CK(cudaMemsetAsync(ctx->d_leafw, 0, sizeof(long long) * kLeafWords * W_ub, ctx->st));
            CK(cudaMemsetAsync(ctx->d_nleft, 0, sizeof(long long) * W_ub, ctx->st));
        }
        TRY(launch(ctx, k_leaf_totals, dim3(tiles_ub), dim3(kPartThreads), 0, ctx->st, ctx->d_xb, ctx->n, ctx->d_rows, ctx->d_tmp,
                                                              ctx->d_ptask, lvl_cnt,
                                                              ints(ctx, I_TILES), ctx->d_q, ctx->d_leafw,
                                                              ctx->d_nleft, (const int32_t *)ctx->d_bigidx,
                                                              (const uint32_t *)ctx->d_topbits,
                                                              ctx->comm ? nullptr : (unsigned *)ints(ctx, I_DONE_LEAF),
                                                              ctx->d_nodes, (const int *)lvl, ctx->S));
        if (ctx->comm) {   // summed over ranks first (one rank: k_leaf_totals' last CTA finished them)
            TRY(allreduce_i64(ctx, ctx->d_leafw, (int64_t)kLeafWords * W_ub));
            TRY(launch(ctx, k_leaf_finish, dim3(1), dim3(256), 0, ctx->st, ctx->d_nodes, lvl, lvl_cnt, ctx->d_leafw,
                       ctx->d_nleft, ctx->S));
        }
        ctx->waves++;
        return GBM_OK;
    }
    const long long *gl = ctx->comm ? nullptr : ctx->d_nleft;   // several ranks: the locally smaller child
    TRY(launch(ctx, k_partition, dim3(tiles_ub), dim3(kPartThreads), 0, ctx->st, (const uint8_t *)ctx->d_xb, ctx->n,
               ctx->d_rows, ctx->d_tmp, (const PartTask *)ctx->d_ptask, (const int *)lvl_cnt,
               (const int *)ints(ctx, I_TILES), ctx->d_tile_st, (unsigned *)ints(ctx, I_TICKET),
               ints(ctx, I_PART_ERR), ctx->d_nleft, (const int32_t *)ctx->d_bigidx,
               (const uint32_t *)ctx->d_topbits, ctx->d_nodes, (const int *)lvl, gl, ctx->d_htask, ctx->d_hprefix,
               (unsigned *)ints(ctx, I_DONE), prune_best_first(P) && !ctx->comm ? 1 : 0,
               (const int *)ints(ctx, I_NODES), P->gamma, (long long)P->min_samples_leaf, P->max_leaves));
    TRY(launch_hist(ctx, rf, lvl_cnt));
    if (ctx->comm) {
        const int cx = std::max(1, (2 * ctx->hist_grid + W_ub - 1) / W_ub);
        unsigned long long *sync = ctx->p2p ? ctx->d_sync : nullptr;
        TRY(launch(ctx, k_stage_left, dim3(cx, W_ub), dim3(256), 0, ctx->st, (const DNode *)ctx->d_nodes,
                   (const int *)lvl, (const int *)lvl_cnt, ctx->d_htask, ctx->p2p ? ctx->d_pst : ctx->d_stage,
                   ctx->pst_stride, ctx->d_lpool, rf.nf, pool_depth(P), sync,
                   (unsigned long long *const *)ctx->d_peer_sync, ctx->p2p_rank, ctx->p2p_n));
        TRY(exchange_stage(ctx, lvl_cnt, W_ub, rf.nf));
        TRY(launch(ctx, k_fill_counts, dim3(1), dim3(256), 0, ctx->st, ctx->d_nodes, (const int *)lvl, lvl_cnt,
                   (const long long *)ctx->d_stage, rf.nf, sync, ctx->p2p_n));
    }
    TRY(launch(ctx, k_split_bins<false>, dim3(rf.nf, W_ub), dim3(kSplitThreads), 0, ctx->st,
        (const DNode *)ctx->d_nodes, (const int *)lvl, (const int *)lvl_cnt, (const HistTask *)ctx->d_htask,
        ctx->d_stage, ctx->d_pool, rf.nf, (const int32_t *)ctx->d_fidx, (const int32_t *)ctx->d_counts,
        (const uint8_t *)(ctx->nan_dir ? ctx->d_nanf : nullptr), ctx->S, P->reg_lambda, P->min_child_weight,
        (long long)P->min_samples_leaf, P->max_depth, pool_depth(P), ctx->d_fbest));
    TRY(launch_close(ctx, rf, P, false, lvl, lvl_cnt, next, next_cnt, next ? np : NextPlan()));
    ctx->waves++;
    return GBM_OK;
}

// Node table -> host (one copy + sync).
int fetch_nodes(gbm_ctx *ctx) {
    CK(cudaMemcpyAsync(ctx->h_ints, ctx->d_ints, sizeof(int) * I_COUNT, cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaMemcpyAsync(ctx->h_nodes, ctx->d_nodes, sizeof(DNode) * ctx->nmax, cudaMemcpyDeviceToHost, ctx->st));
    if (ctx->p2p)
        CK(cudaMemcpyAsync(&ctx->slot[ctx->cur_slot].h_loss[1], ctx->d_sync + ctx->p2p_n + kSyncErr,
                           sizeof(unsigned long long), cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    TRY(p2p_check(ctx, ctx->cur_slot));
    if (ctx->h_ints[I_PART_ERR])
        return fail(ctx, GBM_ERR_STATE, "internal: a partition or compaction tile's wait for its predecessors ran out");
    if (ctx->profiling) TRY(collect_slot_timing(ctx, ctx->cur_slot));
    return GBM_OK;
}

// Expand the given nodes now (the replay needs one that speculation skipped).
int expand_now(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, const std::vector<int> &ids) {
    int W = (int)ids.size();
    if (W == 0) return GBM_OK;
    if (W > ctx->stage_slots) W = ctx->stage_slots;
    if (ctx->h_ints[I_NODES] + 2 * W > ctx->nmax)
        return fail(ctx, GBM_ERR_STATE, "tree node table full (%d nodes)", ctx->nmax);
    for (int k = 0; k < W; k++) ctx->h_list[k] = ids[k];
    ctx->h_list[ctx->stage_slots] = W;
    CK(cudaMemcpyAsync(ctx->d_lvl[0], ctx->h_list, sizeof(int) * W, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ints(ctx, I_LVL0), &ctx->h_list[ctx->stage_slots], sizeof(int), cudaMemcpyHostToDevice,
                       ctx->st));
    TRY(launch_level(ctx, rf, P, ctx->d_lvl[0], ints(ctx, I_LVL0), nullptr, nullptr, W, false, false, NextPlan(),
                     1 << 20));
    return fetch_nodes(ctx);
}

// ---- host tree ------------------------------------------------------------------

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
    int node = 0;      // tree node id (reference numbering)
    int nid = -1;      // device node table index
    int depth = 0, feat = -1, bin = 0, nan_right = 0;
    double gain = -1.0, val = 0.0;
    bool active = false;
};

int replay_leafwise(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, HostTree &T) {
    const int max_leaves = P->max_leaves;
    const int MAXC = max_leaves + 2;
    const double lam = P->reg_lambda, mcw = P->min_child_weight, gamma = P->gamma;
    const long long msl = P->min_samples_leaf;
    T.init(2 * max_leaves + 2);
    const DNode *nd = ctx->h_nodes;
    int node_count = 0;
    int root = node_count++;
    double root_val = -nd[0].G / (nd[0].H + lam);
    if (nd[0].n < msl || nd[0].H < mcw || nd[0].feat < 0) {   // E:575-579, E:634-638
        T.tf[root] = -1; T.tv[root] = root_val; T.nc = node_count;
        return GBM_OK;
    }
    std::vector<Cand> c(MAXC);
    c[0].node = root; c[0].nid = 0; c[0].depth = 0; c[0].gain = nd[0].gain; c[0].feat = nd[0].feat;
    c[0].bin = nd[0].bin; c[0].nan_right = nd[0].nan_right; c[0].val = root_val; c[0].active = true;
    int n_splits = 0;
    while (n_splits < max_leaves - 1) {
        int ci = -1;
        double bg = gamma;
        for (int s = 0; s < MAXC; s++)
            if (c[s].active && c[s].feat >= 0 && c[s].gain > bg) { bg = c[s].gain; ci = s; }
        if (ci < 0) break;
        if (!nd[c[ci].nid].expanded) {
            // expand the best unexpanded candidates now, in selection order
            std::vector<int> order;
            for (int s = 0; s < MAXC; s++)
                if (c[s].active && c[s].feat >= 0 && c[s].gain > gamma && !nd[c[s].nid].expanded) order.push_back(s);
            std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return c[a].gain > c[b].gain; });
            int budget = std::min<int>((int)order.size(), max_leaves - 1 - n_splits);
            std::vector<int> ids;
            for (int q = 0; q < budget; q++) ids.push_back(c[order[q]].nid);
            TRY(expand_now(ctx, rf, P, ids));
            nd = ctx->h_nodes;
            if (!nd[c[ci].nid].expanded) return fail(ctx, GBM_ERR_STATE, "internal: node not expanded");
        }
        Cand &pc = c[ci];
        const DNode &pn = nd[pc.nid];
        int cur = pc.node;
        long long gnl = nd[pn.kid0].n, gnr = nd[pn.kid1].n;
        if (gnl < msl || gnr < msl) {                       // E:678-683
            T.tf[cur] = -1; T.tv[cur] = pc.val; pc.active = false;
            continue;
        }
        int lid = node_count++, rid = node_count++;
        T.tf[cur] = pc.feat; T.tt[cur] = pc.bin | ((int64_t)pc.nan_right << 32); T.tl[cur] = lid; T.tr[cur] = rid;
        T.tv[cur] = pc.val; T.sg[cur] = pc.gain;
        n_splits++;
        int nd_depth = pc.depth + 1;
        if (nd_depth < P->max_depth) {   // the last level builds no histogram
            const DNode &sm = nd[gnl <= gnr ? pn.kid0 : pn.kid1];
            ctx->alg_bytes += (double)(sm.end - sm.begin) * (rf.nf + 8);
            ctx->hist_updates += (double)(sm.end - sm.begin) * rf.upd_per_row;
        }
        bool left_small = gnl <= gnr;
        int ss = -1, sl = -1;                               // E:712-720
        for (int s = 0; s < MAXC; s++) {
            if (s != ci && !c[s].active) {
                if (ss < 0) ss = s; else if (sl < 0) { sl = s; break; }
            }
        }
        c[ci].active = false;
        int kids[2] = {pn.kid0, pn.kid1};
        for (int pass = 0; pass < 2; pass++) {
            int side = (pass == 0) == left_small ? 0 : 1;   // 0 = left
            const DNode &k = nd[kids[side]];
            Cand &x = c[pass == 0 ? ss : sl];
            x = Cand();
            x.node = side == 0 ? lid : rid;
            x.nid = kids[side];
            x.depth = nd_depth;
            x.val = -k.G / (k.H + lam);
            x.feat = k.feat;                    // -1 unless n >= msl, H >= mcw, depth < max_depth (E:775-777)
            x.bin = k.feat >= 0 ? k.bin : 0;
            x.nan_right = k.feat >= 0 ? k.nan_right : 0;
            x.gain = k.feat >= 0 ? k.gain : -1.0;
            x.active = true;
        }
    }
    for (int s = 0; s < MAXC; s++)
        if (c[s].active) { T.tf[c[s].node] = -1; T.tv[c[s].node] = c[s].val; }
    T.nc = node_count;
    return GBM_OK;
}

// Depth-wise DFS builder (E:233-508): node ids in the reference's stack
// order (the larger child pushed first, the smaller popped first).
int replay_depthwise(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, HostTree &T) {
    const double lam = P->reg_lambda;
    const long long msl = P->min_samples_leaf;
    const int D = P->max_depth;
    T.init((1 << (D + 1)) - 1);
    // every node with a split is expanded (unless the node capacity cut a level)
    for (int guard = 0; guard < 64; guard++) {
        std::vector<int> todo;
        int cnt = ctx->h_ints[I_NODES];
        for (int i = 0; i < cnt; i++)
            if (ctx->h_nodes[i].feat >= 0 && !ctx->h_nodes[i].expanded) todo.push_back(i);
        if (todo.empty()) break;
        TRY(expand_now(ctx, rf, P, todo));
    }
    const DNode *nd = ctx->h_nodes;
    int node_count = 0;
    struct SE { int nid, tid; };
    std::vector<SE> stack;
    stack.push_back({0, node_count++});
    while (!stack.empty()) {
        SE e = stack.back();
        stack.pop_back();
        const DNode &x = nd[e.nid];
        double val = -x.G / (x.H + lam);
        bool split = x.feat >= 0 && x.expanded && nd[x.kid0].n >= msl && nd[x.kid1].n >= msl;
        if (!split) { T.tf[e.tid] = -1; T.tv[e.tid] = val; continue; }
        int lid = node_count++, rid = node_count++;
        long long gl = nd[x.kid0].n, gr = nd[x.kid1].n;
        if (x.depth + 1 < D) {
            const DNode &sm = nd[gl <= gr ? x.kid0 : x.kid1];
            ctx->alg_bytes += (double)(sm.end - sm.begin) * (rf.nf + 8);
            ctx->hist_updates += (double)(sm.end - sm.begin) * rf.upd_per_row;
        }
        T.tf[e.tid] = x.feat; T.tt[e.tid] = x.bin | ((int64_t)x.nan_right << 32); T.tl[e.tid] = lid; T.tr[e.tid] = rid;
        T.tv[e.tid] = val; T.sg[e.tid] = x.gain;
        if (gl <= gr) {
            stack.push_back({x.kid1, rid});   // larger pushed first
            stack.push_back({x.kid0, lid});   // smaller popped first
        } else {
            stack.push_back({x.kid0, lid});
            stack.push_back({x.kid1, rid});
        }
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
    int ntile = (int)((ctx->n + kCompTile - 1) / kCompTile);
    for (int q = 0; q < 2; q++) {
        TRY(dalloc(ctx, &ctx->d_maskP[q], (size_t)ctx->n));
        TRY(dalloc(ctx, &ctx->d_rowsP[q], (size_t)ctx->n));
        TRY(dalloc(ctx, &ctx->d_tmpP[q], (size_t)ctx->n));
        TRY(dalloc(ctx, &ctx->d_compP[q], (size_t)ntile + 1));
        CK(cudaMemsetAsync(ctx->d_compP[q], 0, sizeof(unsigned long long) * ((size_t)ntile + 1), ctx->st));
        TRY(dalloc(ctx, &ctx->d_totalP[q], 1));
    }
    use_parity(ctx, 0);
    TRY(dalloc(ctx, &ctx->d_count64, 1));
    TRY(dalloc(ctx, &ctx->d_blist, (size_t)ctx->nblk + 1));   // blist | nb
    TRY(dalloc(ctx, &ctx->d_fbi, (size_t)ctx->p));
    TRY(dalloc(ctx, &ctx->d_fpos, (size_t)ctx->nblk * kBlk));
    TRY(dalloc(ctx, &ctx->d_ints, (size_t)I_COUNT));
    TRY(halloc(ctx, &ctx->h_ints, (size_t)I_COUNT));
    int init[I_COUNT] = {1, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    CK(cudaMemcpyAsync(ctx->d_ints, init, sizeof init, cudaMemcpyHostToDevice, ctx->st));
    TRY(dalloc(ctx, &ctx->d_tree, 1));
    TRY(dalloc(ctx, &ctx->d_leaf, (size_t)ctx->n));
    ctx->upd_blocks = grid_for(ctx->n, kUpdThreads, 148 * 8);
    TRY(dalloc(ctx, &ctx->d_loss_part, (size_t)ctx->upd_blocks));
    TRY(dalloc(ctx, &ctx->d_loss, 1));
    TRY(halloc(ctx, &ctx->h_loss, 1));
    TRY(halloc(ctx, &ctx->h_mask, (size_t)ctx->n));
    ctx->tile_cap = 0;
    return sync_stream(ctx);
}

int check_tree_args(gbm_ctx *ctx, int32_t nfeat, const gbm_params *P, const gbm_tree_out *out) {
    if (nfeat <= 0 || nfeat > ctx->p) return fail(ctx, GBM_ERR_ARG, "nfeat=%d out of range", nfeat);
    if (P->max_leaves < 2 && P->grow_policy == 0) return fail(ctx, GBM_ERR_ARG, "max_leaves must be >= 2");
    if (P->max_depth <= 0) return fail(ctx, GBM_ERR_ARG, "max_depth must be > 0");
    if (P->grow_policy == 1 && P->max_depth > 7)
        return fail(ctx, GBM_ERR_UNSUPPORTED, "depth-wise trees deeper than 7 are not supported");
    if (P->grow_policy == 0 && P->max_leaves > 127)
        return fail(ctx, GBM_ERR_UNSUPPORTED, "max_leaves > 127 is not supported");
    if (P->grow_policy == 0 && P->max_depth > 24)
        return fail(ctx, GBM_ERR_UNSUPPORTED, "max_depth > 24 is not supported");
    int need = P->grow_policy == 0 ? 2 * P->max_leaves + 2 : (1 << (P->max_depth + 1)) - 1;
    if (out->capacity < need) return fail(ctx, GBM_ERR_ARG, "tree capacity %d < %d", out->capacity, need);
    if (P->nan_direction && !P->nan_bin_id)
        return fail(ctx, GBM_ERR_ARG, "nan_direction needs nan_bin_id (the reference's _nan_bin_id)");
    return GBM_OK;
}

int tree_need(const gbm_params *P) {
    return P->grow_policy == 0 ? 2 * P->max_leaves + 2 : (1 << (P->max_depth + 1)) - 1;
}

// Enqueue the in-bag compaction and the level-wise growth; the round's
// in-bag mask is on the device and its feature tables are staged.
// In-bag mask -> ascending row list of the root (row buffer 0) and its count.
int enqueue_compaction(gbm_ctx *ctx, cudaStream_t s) {
    int ntile = (int)((ctx->n + kCompTile - 1) / kCompTile);
    return launch(ctx, k_compact_rows, dim3(ntile), dim3(kCompThreads), 0, s, (const uint8_t *)ctx->d_mask, ctx->n,
                  ctx->d_rows, ctx->d_total, ctx->d_comp, (unsigned *)(ctx->d_comp + ntile), ints(ctx, I_PART_ERR));
}

// `compacted`: the root's row list was already built (stage_sample, on the
// sampler stream); otherwise it is built here from d_mask.
int enqueue_grow(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, bool compacted) {
    TRY(flush_l2(ctx));
    if (!compacted) TRY(enqueue_compaction(ctx, ctx->st));
    if (ctx->comm) TRY(gbm_comm_check_alive(ctx->comm, ctx->timeout_ms, ctx->err));
    const int D = P->max_depth;
    auto plan_of = [&](int L) {
        NextPlan np;
        if (L < D) {
            np.W_ub = std::min(level_width(P, L), ctx->stage_slots);
            np.last = L == D - 1;
        }
        return np;
    };
    TRY(launch_root(ctx, rf, P, plan_of(0)));
    int cur = 0;
    for (int L = 0; L < D; L++) {
        const NextPlan me = plan_of(L);
        TRY(launch_level(ctx, rf, P, ctx->d_lvl[cur], ints(ctx, I_LVL0 + cur), ctx->d_lvl[1 - cur],
                         ints(ctx, I_LVL0 + 1 - cur), me.W_ub, me.last, true, plan_of(L + 1), L + 1));
        cur = 1 - cur;
    }
    // this parity's row lists and packed blocks are free: the round two
    // places on may overwrite them
    TRY(record_ev(ctx, ctx->rows_free, ctx->st));
    if (ctx->p2p)   // the exchange's error word travels with the round
        CK(cudaMemcpyAsync(&ctx->slot[ctx->cur_slot].h_loss[1], ctx->d_sync + ctx->p2p_n + kSyncErr,
                           sizeof(unsigned long long), cudaMemcpyDeviceToHost, ctx->st));
    return GBM_OK;
}

// The host replay, for best-first trees deeper than kSpecDepth: one node
// table fetch, on-demand expansion of what the level ranking left out,
// post-prune and monotone clipping.
int replay_on_host(gbm_ctx *ctx, const RoundFeat &rf, const gbm_params *P, HostTree &T) {
    TRY(fetch_nodes(ctx));
    ctx->alg_bytes += (double)(ctx->h_nodes[0].end - ctx->h_nodes[0].begin) * (rf.nf + 8);
    ctx->hist_updates += (double)(ctx->h_nodes[0].end - ctx->h_nodes[0].begin) * rf.upd_per_row;
    ctx->hist_rows += ctx->h_nodes[0].end;
    auto t_rep = std::chrono::steady_clock::now();
    double sync_before = ctx->host_sync_ms;
    if (P->grow_policy == 0) TRY(replay_leafwise(ctx, rf, P, T));
    else TRY(replay_depthwise(ctx, rf, P, T));
    ctx->host_replay_ms += ms_since(t_rep) - (ctx->host_sync_ms - sync_before);
    post_prune(T, P->gamma);
    enforce_monotone(T, P->monotone);
    return GBM_OK;
}

// Monotone constraints of this call -> the device (before any round of the
// call is queued; every earlier call has finished).
int stage_mono(gbm_ctx *ctx, const gbm_params *P) {
    ctx->nan_dir = P->nan_direction != 0;
    if (ctx->nan_dir) {   // which features' bin 0 is a NaN bin
        for (int j = 0; j < ctx->p; j++) ctx->h_nanf[j] = P->nan_bin_id[j] == 0 ? 1 : 0;
        CK(cudaMemcpyAsync(ctx->d_nanf, ctx->h_nanf, (size_t)ctx->p, cudaMemcpyHostToDevice, ctx->st));
    }
    if (!P->monotone) return GBM_OK;
    std::memcpy(ctx->h_mono, P->monotone, sizeof(int32_t) * ctx->p);
    CK(cudaMemcpyAsync(ctx->d_mono, ctx->h_mono, sizeof(int32_t) * ctx->p, cudaMemcpyHostToDevice, ctx->st));
    return GBM_OK;
}

// Enqueue the device replay: the tree into d_tout (host layout) and d_tree
// (the F update's layout).
int enqueue_replay(gbm_ctx *ctx, const gbm_params *P) {
    RParams R;
    R.lam = P->reg_lambda;
    R.gamma = P->gamma;
    R.mcw = P->min_child_weight;
    R.msl = P->min_samples_leaf;
    R.max_depth = P->max_depth;
    R.max_leaves = P->max_leaves;
    R.policy = P->grow_policy;
    R.has_mono = P->monotone != nullptr;
    R.part_err = ints(ctx, I_PART_ERR);
    size_t smem = sizeof(RNode) * (size_t)ctx->nmax;
    if (P->grow_policy == 0)
        TRY(launch(ctx, k_replay_leaf, dim3(1), dim3(kReplayLoaders), smem, ctx->st, ctx->d_nodes, ints(ctx, I_NODES), R,
                   ctx->d_mono, ctx->d_tout, ctx->d_tree));
    else
        TRY(launch(ctx, k_replay_depth, dim3(1), dim3(kReplayLoaders), smem, ctx->st, ctx->d_nodes, ints(ctx, I_NODES), R, ctx->d_mono, ctx->d_tout,
                                                 ctx->d_tree));
    return GBM_OK;
}

// Enqueue the F update, the next gradients and the train loss of the tree
// in d_tree; the loss goes to the slot's pinned buffer.
int enqueue_update(gbm_ctx *ctx, const gbm_params *P, bool want_leaf, double *h_loss) {
    double scale = std::ldexp(1.0, ctx->S);
    TRY(launch(ctx, k_update, dim3(ctx->upd_blocks), dim3(kUpdThreads), 0, ctx->st, 
        ctx->d_tree, ctx->d_xb, ctx->n, ctx->d_y, ctx->w[0], ctx->w[1], P->learning_rate, scale, ctx->d_F,
        ctx->d_q, want_leaf ? ctx->d_leaf : nullptr, ctx->d_loss_part, (unsigned *)ints(ctx, I_DONE_UPD),
        ctx->d_loss, (const int32_t *)ctx->d_bigidx, (const uint32_t *)ctx->d_topbits));
    if (ctx->comm) TRY(allreduce_f64(ctx, ctx->d_loss, 1));
    CK(cudaMemcpyAsync(h_loss, ctx->d_loss, sizeof(double), cudaMemcpyDeviceToHost, ctx->st));
    return GBM_OK;
}

// Wait (bounded, watching the communicator) for a slot's round to finish.
int wait_slot(gbm_ctx *ctx, int si) {
    auto t0 = std::chrono::steady_clock::now();
    int rc = gbm_comm_wait_event(ctx->comm, ctx->slot[si].done, ctx->timeout_ms, ctx->err);
    ctx->host_sync_ms += ms_since(t0);
    return rc;
}

void write_tree_dev(const TreeOut &T, int need, gbm_tree_out *out) {
    for (int k = 0; k < need; k++) {
        bool in = k < 256;
        out->tf[k] = in ? T.tf[k] : -1;
        out->tt[k] = in ? T.tt[k] : 0;
        out->tv[k] = in ? T.tv[k] : 0.0;
        out->tl[k] = in ? T.tl[k] : -1;
        out->tr[k] = in ? T.tr[k] : -1;
        out->sg[k] = in ? T.sg[k] : 0.0;
        if (out->nan_right) out->nan_right[k] = in ? T.nr[k] : 0;
    }
    out->n_nodes = T.nc;
}

// A finished slot -> the caller's tree and loss, and the statistics.
// A device-replayed tree record: its status, the statistics, the caller's arrays.
int take_tree(gbm_ctx *ctx, const TreeOut &T, double upd_per_row, int nf, const gbm_params *P, gbm_tree_out *out) {
    if (T.status == 3)
        return fail(ctx, GBM_ERR_STATE, "internal: a partition or compaction tile's wait for its predecessors ran out");
    if (T.status != 0) return fail(ctx, GBM_ERR_STATE, "internal: the device replay reached an unexpanded node");
    ctx->alg_bytes += (double)T.alg_rows * (nf + 8);
    ctx->hist_updates += (double)T.alg_rows * upd_per_row;
    ctx->hist_rows += T.root_rows;
    write_tree_dev(T, tree_need(P), out);
    return GBM_OK;
}

int harvest(gbm_ctx *ctx, int si, int nf, const gbm_params *P, gbm_tree_out *out, double *train_loss) {
    if (ctx->profiling) TRY(collect_slot_timing(ctx, si));
    TRY(p2p_check(ctx, si));
    TRY(take_tree(ctx, *ctx->slot[si].h_tout, ctx->slot[si].upd_per_row, nf, P, out));
    if (train_loss) *train_loss = -ctx->slot[si].h_loss[0] / (double)ctx->n_global;
    return GBM_OK;
}

void write_tree(const HostTree &T, int need, gbm_tree_out *out) {
    for (int k = 0; k < need; k++) {
        bool in = k < (int)T.tf.size();
        out->tf[k] = in ? T.tf[k] : -1;
        out->tt[k] = in ? (T.tt[k] & 0xffffffffll) : 0;   // the NaN direction rides in bit 32
        if (out->nan_right) out->nan_right[k] = in ? (int32_t)(T.tt[k] >> 32) : 0;
        out->tv[k] = in ? T.tv[k] : 0.0;
        out->tl[k] = in ? T.tl[k] : -1;
        out->tr[k] = in ? T.tr[k] : -1;
        out->sg[k] = in ? T.sg[k] : 0.0;
    }
    out->n_nodes = T.nc;
}


// Buffers, slots and the monotone table for a call's rounds.
int prepare_round(gbm_ctx *ctx, int nf, const gbm_params *P) {
    TRY(ensure_round_buffers(ctx, nf, P));
    TRY(ensure_slots(ctx));
    // staging histograms start every call at zero (each use zeroes what it read)
    CK(cudaMemsetAsync(ctx->d_stage, 0, sizeof(long long) * (size_t)ctx->stage_slots * slot_words_for(ctx->nf_cap),
                       ctx->st));
    use_parity(ctx, 0);   // the one-round calls use slot 0's buffers; begin_round picks a ring slot's
    return stage_mono(ctx, P);
}

// The sampler's next round (host side): its row swap targets into slot
// si's pinned buffer and its features into feat_buf.  A sampler at its
// first round is bound here: the previous permutation becomes arange(N).
// Slot si must be the round's index modulo kRing (the permutation chain).
int take_sample(gbm_ctx *ctx, int si, gbm_sampler *sampler, int64_t row_offset) {
    gbm_ctx::Slot &s = ctx->slot[si];
    const int64_t N = gbm_sampler_rows(sampler);
    const bool rows_on = gbm_sampler_shuffles_rows(sampler) != 0;
    const int64_t r = gbm_sampler_taken(sampler);
    constexpr int R = gbm_ctx::kRing;
    if (row_offset + ctx->n > N) return fail(ctx, GBM_ERR_ARG, "rows %lld.. exceed the sampler's %lld rows",
                                             (long long)row_offset, (long long)N);
    if (si != (int)(r % R)) return fail(ctx, GBM_ERR_STATE, "internal: slot %d for round %lld", si, (long long)r);
    if (rows_on) TRY(ensure_shuffle(ctx, N));
    if (ctx->samp != sampler || ctx->samp_taken != r) {
        if (r != 0)
            return fail(ctx, GBM_ERR_STATE, "the sampler is at round %lld, which this engine did not draw",
                        (long long)r);
        ctx->samp = sampler;
        ctx->samp_taken = 0;
        if (rows_on) TRY(launch(ctx, k_iota, dim3(grid_for(N, 256)), dim3(256), 0, ctx->cst, ctx->d_perm[R - 1], N));
    }
    ctx->feat_buf.resize((size_t)gbm_sampler_n_feat(sampler));
    s.h_round[0] = (long long)r;   // the round a throughput-mode sampler hashes its rows with
    auto t_s = std::chrono::steady_clock::now();
    int rc = gbm_sampler_take_targets(sampler, s.h_tg, ctx->feat_buf.data());
    ctx->host_sample_ms += ms_since(t_s);
    if (rc != GBM_OK) return fail(ctx, rc, "the sampler cannot feed an engine (already used for host draws?)");
    ctx->samp_taken++;
    return GBM_OK;
}

// The round's shuffle (composed into the permutation), this rank's in-bag
// mask and the root's row list, on the sampler stream (cst); ends with
// slot si's `copied` event, which the engine stream waits for.
// Throughput-mode rows of a sampler (gbm_sampler_create_device), or none.
struct DevRows {
    bool on = false;
    uint64_t seed = 0, thr = 0;
};

DevRows dev_rows_of(const gbm_sampler *sampler) {
    DevRows d;
    d.on = gbm_sampler_device_rows(sampler, &d.seed, &d.thr) != 0;
    return d;
}

int enqueue_sample(gbm_ctx *ctx, int si, int64_t N, int64_t m, bool rows_on, int64_t row_offset, int nf,
                   const DevRows &dr) {
    gbm_ctx::Slot &s = ctx->slot[si];
    constexpr int R = gbm_ctx::kRing;
    int32_t *pout = nullptr;
    // Everything this round writes here -- its packed feature blocks
    // (d_xc[si & 1]), its mask, root row list and compaction scratch (the
    // parity set of use_parity) -- was last used by the round two places
    // back: wait for that round's last level, then build them while the
    // previous round grows.
    TRY(wait_ev(ctx, ctx->cst, ctx->rows_free));
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    if (ctx->profiling) {
        TRY(timing_pair(ctx, 3, t0, t1));
        TRY(record_ev(ctx, t0, ctx->cst));
    }
    s.xc_on_cst = nf > 0 && compact_hist(ctx);
    if (s.xc_on_cst) {
        CK(cudaMemcpyAsync(s.d_fidx_c, s.h_feat, sizeof(int32_t) * nf, cudaMemcpyHostToDevice, ctx->cst));
        TRY(enqueue_pack(ctx, ctx->cst, s.d_fidx_c, nf, ctx->d_xc[si & 1]));
    }
    if (rows_on) {
        int32_t *pin = ctx->d_perm[(si + R - 1) % R];
        pout = ctx->d_perm[si];
        CK(cudaMemcpyAsync(s.d_tg, s.h_tg, sizeof(int32_t) * (size_t)(N - 1), cudaMemcpyHostToDevice, ctx->cst));
        CK(cudaMemsetAsync(ctx->d_head, 0xff, sizeof(int32_t) * (size_t)N, ctx->cst));
        TRY(launch(ctx, k_shuf_link, dim3(grid_for(N - 1, 256)), dim3(256), 0, ctx->cst, s.d_tg, N, ctx->d_head,
                   ctx->d_nxt));
        TRY(launch(ctx, k_shuf_min, dim3(grid_for(N, 256)), dim3(256), 0, ctx->cst, s.d_tg, N, ctx->d_head,
                   ctx->d_nxt, ctx->d_m, ctx->d_mp));
        TRY(launch(ctx, k_shuf_compose, dim3(grid_for(N, 256)), dim3(256), 0, ctx->cst, s.d_tg, N, ctx->d_m,
                   ctx->d_mp, pin, pout));
    }
    // The mask and root row list: with at most kEarlyRootRows rows on this
    // rank they are built during the previous round's levels (config 4,
    // 1M rows: 0.758 -> 0.741 ms per round); with more, after them (config
    // 5, 10M rows: 7.90 against 8.85 ms per round when built early).
    if (ctx->n > kEarlyRootRows) TRY(wait_ev(ctx, ctx->cst, ctx->rows_freeP[(si + 1) & 1]));
    if (dr.on) {   // throughput mode: this rank's rows from the hash of (seed, round, global row)
        CK(cudaMemcpyAsync(s.d_round, s.h_round, sizeof(long long), cudaMemcpyHostToDevice, ctx->cst));
        TRY(launch(ctx, k_mask_hash, dim3(grid_for(ctx->n, 256)), dim3(256), 0, ctx->cst, ctx->d_mask, ctx->n,
                   row_offset, dr.seed, dr.thr, (const long long *)s.d_round));
    } else if (rows_on) {
        CK(cudaMemsetAsync(ctx->d_mask, 0, (size_t)ctx->n, ctx->cst));
        TRY(launch(ctx, k_mask_from_rows, dim3(grid_for(m, 256)), dim3(256), 0, ctx->cst, pout, m, row_offset,
                   ctx->n, ctx->d_mask));
    } else {   // sample_idx is every row (E:2508-2509)
        CK(cudaMemsetAsync(ctx->d_mask, 1, (size_t)ctx->n, ctx->cst));
    }
    TRY(enqueue_compaction(ctx, ctx->cst));
    if (t1) TRY(record_ev(ctx, t1, ctx->cst));
    TRY(record_ev(ctx, s.copied, ctx->cst));
    return GBM_OK;
}

// Sizes, bin counts and the training matrix buffer for n rows x p
// features; features of 257 bins get their big index and zeroed top bits.
int begin_bins(gbm_ctx *ctx, int64_t n, int32_t p, const int32_t *bin_counts) {
    if (!ctx || !bin_counts || n <= 0 || p <= 0 || n > 0x7fffffffLL) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    for (int j = 0; j < p; j++)
        if (bin_counts[j] < 1 || bin_counts[j] > kBins + 1)
            return fail(ctx, GBM_ERR_UNSUPPORTED, "feature %d has %d bins; the device path holds 1..257 bins",
                        j, bin_counts[j]);
    CK(cudaSetDevice(ctx->dev));
    ctx->n = n; ctx->p = p; ctx->nblk = (p + kBlk - 1) / kBlk;
    ctx->slots_ready = false;
    ctx->have_bins = ctx->have_labels = ctx->have_labels_mc = ctx->have_targets = false;
    ctx->counts.assign(bin_counts, bin_counts + p);
    TRY(dalloc(ctx, &ctx->d_xb, (size_t)ctx->nblk * n * kBlk));
    if (compact_hist(ctx))
        for (auto &b : ctx->d_xc) TRY(dalloc(ctx, &b, (size_t)ctx->nblk * n * kBlk));
    TRY(dalloc(ctx, &ctx->d_counts, (size_t)p));
    CK(cudaMemcpyAsync(ctx->d_counts, bin_counts, sizeof(int32_t) * p, cudaMemcpyHostToDevice, ctx->st));
    std::vector<int32_t> bigidx((size_t)p, -1);
    ctx->bigfeat.clear();
    for (int j = 0; j < p; j++)
        if (bin_counts[j] > kBins) {
            bigidx[(size_t)j] = (int32_t)ctx->bigfeat.size();
            ctx->bigfeat.push_back(j);
        }
    ctx->nbig = (int)ctx->bigfeat.size();
    TRY(dalloc(ctx, &ctx->d_bigidx, (size_t)p));
    CK(cudaMemcpy(ctx->d_bigidx, bigidx.data(), sizeof(int32_t) * p, cudaMemcpyHostToDevice));
    if (ctx->nbig) {
        const size_t words = (size_t)ctx->nbig * (size_t)((n + 31) >> 5);
        TRY(dalloc(ctx, &ctx->d_topbits, words));
        CK(cudaMemsetAsync(ctx->d_topbits, 0, sizeof(uint32_t) * words, ctx->st));
        TRY(dalloc(ctx, &ctx->d_bigfeat, (size_t)ctx->nbig));
        CK(cudaMemcpy(ctx->d_bigfeat, ctx->bigfeat.data(), sizeof(int32_t) * ctx->nbig, cudaMemcpyHostToDevice));
        TRY(dalloc(ctx, &ctx->d_topoff, (size_t)ctx->nbig + 1));
    }
    return GBM_OK;
}

// The ascending row lists of the top bits (k_hist_top's input).
int build_top_lists(gbm_ctx *ctx) {
    if (!ctx->nbig) return GBM_OK;
    const int64_t wp = (ctx->n + 31) >> 5;
    TRY(launch(ctx, k_top_list<false>, dim3(ctx->nbig), dim3(256), 0, ctx->st, (const uint32_t *)ctx->d_topbits, wp,
               ctx->n, ctx->d_topoff, (const int32_t *)nullptr, (int32_t *)nullptr));
    std::vector<int32_t> off((size_t)ctx->nbig + 1, 0);
    CK(cudaMemcpyAsync(off.data() + 1, ctx->d_topoff, sizeof(int32_t) * ctx->nbig, cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    for (int b = 0; b < ctx->nbig; b++) off[(size_t)b + 1] += off[(size_t)b];
    TRY(dalloc(ctx, &ctx->d_toprows, (size_t)std::max(1, off[(size_t)ctx->nbig])));
    CK(cudaMemcpyAsync(ctx->d_topoff, off.data(), sizeof(int32_t) * (ctx->nbig + 1), cudaMemcpyHostToDevice, ctx->st));
    TRY(launch(ctx, k_top_list<true>, dim3(ctx->nbig), dim3(256), 0, ctx->st, (const uint32_t *)ctx->d_topbits, wp,
               ctx->n, (int32_t *)nullptr, (const int32_t *)ctx->d_topoff, ctx->d_toprows));
    return sync_stream(ctx);
}

// Top bits from the uint16 upload's element indices (row * p + feature) of
// ids above 255: the features of 257 bins read them as bin 256; every
// other feature's clamp to bin_count - 1 already holds them.
int set_top_bits(gbm_ctx *ctx, const std::vector<int64_t> &wide, int32_t p, const std::vector<int32_t> &bigidx,
                 int64_t rows, uint32_t *bits) {
    std::vector<int64_t> pairs;
    for (int64_t e : wide) {
        const int32_t b = bigidx[(size_t)(e % p)];
        if (b >= 0) {
            pairs.push_back(e / p);
            pairs.push_back(b);
        }
    }
    if (pairs.empty()) return GBM_OK;
    const int64_t m = (int64_t)pairs.size() / 2;
    TRY(dalloc(ctx, &ctx->d_toppairs, pairs.size()));
    CK(cudaMemcpyAsync(ctx->d_toppairs, pairs.data(), sizeof(int64_t) * pairs.size(), cudaMemcpyHostToDevice,
                       ctx->st));
    TRY(launch(ctx, k_set_topbits, dim3(grid_for(m, 256)), dim3(256), 0, ctx->st, (const int64_t *)ctx->d_toppairs,
               m, (rows + 31) >> 5, bits));
    return sync_stream(ctx);   // the pairs are host memory freed on return
}

// Everything that depends on the bins once they are on the device.
int finish_bins(gbm_ctx *ctx) {
    TRY(sync_stream(ctx));
    TRY(build_top_lists(ctx));
    TRY(alloc_round_fixed(ctx));
    TRY(dalloc(ctx, &ctx->d_y, (size_t)ctx->n));
    TRY(dalloc(ctx, &ctx->d_F, (size_t)ctx->n));
    TRY(dalloc(ctx, &ctx->d_q, (size_t)ctx->n));
    ctx->have_bins = true;
    ctx->have_labels = false;
    return GBM_OK;
}

int ensure_uploads(gbm_ctx *ctx) {
    if (!ctx->stager) ctx->stager = gbmh2d::stager_create();
    if (!ctx->d_upstage) TRY(dalloc(ctx, &ctx->d_upstage, gbmh2d::chunk_bytes()));
    if (!ctx->bw) ctx->bw = gbmbin::work_create();
    return GBM_OK;
}

// Row-major uint8/uint16 ids -> column blocks: rows stream through pinned
// buffers (uint16 narrowed to uint8 on the host, halving the copy), each
// chunk is transposed and clamped to bin_count - 1 on the device.
template <typename T>
int upload_bins_t(gbm_ctx *ctx, const T *xbin, int64_t n, int32_t p, const int32_t *bin_counts) {
    if (!xbin) return GBM_ERR_ARG;
    TRY(begin_bins(ctx, n, p, bin_counts));
    TRY(ensure_uploads(ctx));
    uint8_t *stage = ctx->d_upstage;
    const int nblk = ctx->nblk;
    auto dst = [stage](int64_t, int64_t) { return static_cast<void *>(stage); };
    auto after = [&](int64_t r0, int64_t nr, const void *) -> int {
        k_pack_bins<uint8_t><<<grid_for(nr * nblk, 256), 256, 0, ctx->st>>>(stage, nr, p, r0, n, nblk,
                                                                           ctx->d_counts, ctx->d_xb);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) return 0;
        ctx->err = std::string("k_pack_bins: ") + cudaGetErrorString(e);
        return GBM_ERR_CUDA;
    };
    std::string err;
    const gbmh2d::Pack pk = sizeof(T) == 2 ? gbmh2d::Pack::U16toU8 : gbmh2d::Pack::Copy;
    std::vector<int64_t> wide;   // uint16 ids above 255
    if (gbmh2d::stream_rows(ctx->stager, ctx->st, xbin, n, sizeof(T) * (size_t)p, pk, 0, dst, after, err,
                            ctx->nbig ? &wide : nullptr))
        return fail(ctx, GBM_ERR_CUDA, "bin upload: %s", err.empty() ? ctx->err.c_str() : err.c_str());
    if (!wide.empty()) {
        std::vector<int32_t> bigidx((size_t)p, -1);
        for (int b = 0; b < ctx->nbig; b++) bigidx[(size_t)ctx->bigfeat[(size_t)b]] = b;
        TRY(set_top_bits(ctx, wide, p, bigidx, n, ctx->d_topbits));
    }
    return finish_bins(ctx);
}

}  // namespace

namespace {

// Everything a captured round depends on besides the contents of its
// slot's pinned buffers.
std::string graph_key(const gbm_ctx *ctx, const gbm_params *P, int nf, int64_t N, int64_t m, bool rows_on,
                      int64_t row_offset) {
    char buf[512];
    snprintf(buf, sizeof buf, "%a/%a/%a/%a/%d/%d/%d/%d/%p/%d/%p|%d/%lld/%lld/%lld/%d/%lld|%d/%zu/%llu/%p",
             P->reg_lambda, P->gamma, P->min_child_weight, P->learning_rate, P->min_samples_leaf, P->max_depth,
             P->max_leaves, P->grow_policy, (const void *)P->monotone, P->nan_direction,
             (const void *)P->nan_bin_id, nf, (long long)N, (long long)m,
             (long long)ctx->n, (int)rows_on, (long long)row_offset, (int)ctx->profiling, ctx->flush_bytes,
             ctx->mem_gen, (const void *)ctx->comm);
    return buf;
}

void drop_graphs(gbm_ctx *ctx) {
    for (auto &s : ctx->slot) {
        if (s.g_cst) cudaGraphExecDestroy(s.g_cst);
        if (s.g_st) cudaGraphExecDestroy(s.g_st);
        s.g_cst = s.g_st = nullptr;
    }
    ctx->graph_key.clear();
}

// Capture one stream's part of a round into an executable graph.
template <typename F>
int capture(gbm_ctx *ctx, cudaStream_t st, cudaGraphExec_t *out, F &&enqueue) {
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    ctx->capturing = true;
    int rc = enqueue();
    ctx->capturing = false;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc == GBM_OK && e != cudaSuccess) rc = fail(ctx, GBM_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    if (rc == GBM_OK) {
        e = cudaGraphInstantiate(out, g, 0);
        if (e != cudaSuccess) rc = fail(ctx, GBM_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    }
    if (g) cudaGraphDestroy(g);
    return rc;
}

// Slot si's round as two graphs: the sampler stream's part (targets,
// shuffle, mask, root row list) and the engine stream's (features, growth,
// replay, F update, tree and loss copies).  The host fills the slot's pinned
// buffers before each launch.
int capture_round(gbm_ctx *ctx, int si, int nf, const gbm_params *P, int64_t N, int64_t m, bool rows_on,
                  int64_t row_offset, const DevRows &dr) {
    gbm_ctx::Slot &s = ctx->slot[si];
    const long long l0 = ctx->launches, h0 = ctx->hist_launches, w0 = ctx->waves;
    const double b0 = ctx->comm_bytes;
    ctx->cur_slot = si;
    use_parity(ctx, si & 1);
    s.tused = s.tdone = 0;
    TRY(capture(ctx, ctx->cst, &s.g_cst, [&] { return enqueue_sample(ctx, si, N, m, rows_on, row_offset, nf, dr); }));
    TRY(capture(ctx, ctx->st, &s.g_st, [&] {
        TRY(wait_copied(ctx, s));
        TRY(enqueue_features(ctx, si, nf));
        RoundFeat rf;
        rf.nf = nf;
        TRY(enqueue_grow(ctx, rf, P, true));
        TRY(enqueue_replay(ctx, P));
        TRY(enqueue_update(ctx, P, false, s.h_loss));
        CK(cudaMemcpyAsync(s.h_tout, ctx->d_tout, sizeof(TreeOut), cudaMemcpyDeviceToHost, ctx->st));
        return record_ev(ctx, s.done, ctx->st);
    }));
    s.g_tpairs = s.tused;
    s.g_launches = ctx->launches - l0;
    s.g_hist = ctx->hist_launches - h0;
    s.g_waves = ctx->waves - w0;
    s.g_comm_bytes = ctx->comm_bytes - b0;
    ctx->launches = l0;   // counted when the graphs run
    ctx->hist_launches = h0;
    ctx->waves = w0;
    ctx->comm_bytes = b0;
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
    // Both streams at the default priority: a high-priority engine stream
    // measured slower on config 5 (6.67 -> 8.10 ms per round, the sampler
    // stream's packing then running late into the next round) and the same
    // on config 4 (0.739 against 0.741 ms).
    CK(cudaStreamCreateWithFlags(&ctx->st, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&ctx->cst, cudaStreamNonBlocking));
    for (auto &e : ctx->rows_freeP) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    ctx->rows_free = ctx->rows_freeP[0];
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    ctx->sms = std::max(sms, 1);
    ctx->hist_grid = 2 * ctx->sms;
    if (const char *e = std::getenv("GBM_HIST_COMPACT")) ctx->hist_compact = std::atoi(e) != 0;
    if (const char *e = std::getenv("GBM_HIST_SEG_COST")) ctx->hist_seg_cost = std::max(0, std::atoi(e));
    CK(cudaFuncSetAttribute(k_hist3<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)(kAccV3Words * sizeof(unsigned))));
    CK(cudaFuncSetAttribute(k_hist3<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)(kAccV3Words * sizeof(unsigned))));
    CK(cudaFuncSetAttribute(k_compact_feat, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    // a function attribute is shared by every context of the process: set
    // the largest node-table copy any context may launch with
    CK(cudaFuncSetAttribute(k_replay_leaf, cudaFuncAttributeMaxDynamicSharedMemorySize, kReplaySmemMax));
    CK(cudaFuncSetAttribute(k_replay_depth, cudaFuncAttributeMaxDynamicSharedMemorySize, kReplaySmemMax));
    return GBM_OK;
}

const char *gbm_last_error(const gbm_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

void gbm_ctx_destroy(gbm_ctx *ctx) {
    if (!ctx) return;
    if (ctx->dev >= 0) {
        cudaSetDevice(ctx->dev);
        if (ctx->st) cudaStreamSynchronize(ctx->st);
        if (ctx->cst) cudaStreamSynchronize(ctx->cst);
    }
    drop_graphs(ctx);   // graphs may hold collectives: release them first
    p2p_teardown(ctx, false);
    gbmh2d::stager_destroy(ctx->stager);
    gbmbin::work_destroy(ctx->bw);
    for (auto &s : ctx->slot)
        for (cudaEvent_t e : s.tev) cudaEventDestroy(e);
    if (ctx->comm) gbm_comm_destroy(ctx->comm);
    for (int q = 0; q < 2; q++) {
        void *pq[] = {ctx->d_maskP[q], ctx->d_rowsP[q], ctx->d_tmpP[q], ctx->d_compP[q], ctx->d_totalP[q]};
        for (void *p : pq) if (p) cudaFree(p);
    }
    void *dev_ptrs[] = {ctx->d_xb, ctx->d_xc[0], ctx->d_xc[1], ctx->d_counts, ctx->d_y, ctx->d_F, ctx->d_q,
                        ctx->d_blist, ctx->d_fidx,
                        ctx->d_fpos, ctx->d_pool, ctx->d_lpool, ctx->d_stage, ctx->d_fbest, ctx->d_htask, ctx->d_hprefix,
                        ctx->d_ptask, ctx->d_nleft,
                        ctx->d_count64, ctx->d_nodes, ctx->d_lvl[0], ctx->d_lvl[1], ctx->d_ints, ctx->d_tree,
                        ctx->d_leaf, ctx->d_loss_part, ctx->d_loss, ctx->d_px, ctx->d_pnodes, ctx->d_pvals,
                        ctx->d_poff, ctx->d_pchunk, ctx->d_pdep, ctx->d_pF, ctx->d_pP, ctx->d_tout, ctx->d_mono, ctx->d_flush,
                        ctx->d_head, ctx->d_nxt, ctx->d_m, ctx->d_mp, ctx->d_fbi, 
                        ctx->d_upstage, ctx->d_Fmc, ctx->d_wmc, ctx->d_qmc, ctx->d_yr,
                        ctx->d_gmax_part, ctx->d_gmax, ctx->d_stab, ctx->d_leafw, ctx->d_nanf, ctx->d_bigidx,
                        ctx->d_bigfeat, ctx->d_topoff, ctx->d_toprows, ctx->d_topbits, ctx->d_toppairs,
                        ctx->d_pbigidx, ctx->d_ptopbits};
    for (int32_t *q : ctx->d_perm) if (q) cudaFree(q);
    for (void *p : dev_ptrs) if (p) cudaFree(p);
    void *host_ptrs[] = {ctx->h_nodes, ctx->h_ints, ctx->h_list, ctx->h_loss, ctx->h_mask, ctx->h_mono, ctx->h_nanf,
                         ctx->h_tout_mc};
    for (void *p : host_ptrs) if (p) cudaFreeHost(p);
    for (auto &s : ctx->slot) {
        if (s.d_tg) cudaFree(s.d_tg);
        if (s.d_fidx_c) cudaFree(s.d_fidx_c);
        if (s.d_round) cudaFree(s.d_round);
        if (s.h_round) cudaFreeHost(s.h_round);
        void *hp[] = {s.h_tg, s.h_feat, s.h_fpos, s.h_tout, s.h_loss};
        for (void *p : hp) if (p) cudaFreeHost(p);
        if (s.copied) cudaEventDestroy(s.copied);
        if (s.done) cudaEventDestroy(s.done);
    }
    for (cudaEvent_t e : ctx->mark) if (e) cudaEventDestroy(e);
    if (ctx->st) cudaStreamDestroy(ctx->st);
    if (ctx->cst) cudaStreamDestroy(ctx->cst);
    for (auto &e : ctx->rows_freeP) if (e) cudaEventDestroy(e);
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
    if (ctx->comm) {   // replaced: finish its work and drop the graphs that call it first
        TRY(sync_stream(ctx));
        drop_graphs(ctx);
        TRY(p2p_teardown(ctx, true));
        gbm_comm_destroy(ctx->comm);
        ctx->comm = nullptr;
    }
    ctx->p2p_tried_stride = 0;
    if (nranks == 1) return GBM_OK;
    TRY(gbm_comm_create(&ctx->comm, uid, nranks, rank, ctx->timeout_ms, ctx->err));
    return GBM_OK;
}

int gbm_nccl_unique_id(void *uid_out) { return gbm_comm_unique_id(uid_out); }

int gbm_upload_bins(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p, const int32_t *bin_counts) {
    return upload_bins_t(ctx, xbin, n, p, bin_counts);
}

int gbm_upload_bins_u16(gbm_ctx *ctx, const uint16_t *xbin, int64_t n, int32_t p, const int32_t *bin_counts) {
    return upload_bins_t(ctx, xbin, n, p, bin_counts);
}

// ---- binning on the device ------------------------------------------------------

static int bin_fail(gbm_ctx *ctx, const std::string &err) {
    const bool arg = err.rfind("binning:", 0) == 0;
    return fail(ctx, arg ? GBM_ERR_ARG : GBM_ERR_CUDA, "%s", err.c_str());
}

int gbm_bin_edges(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype, int32_t n_bins,
                  const uint8_t *is_cat, double *edges_out, int32_t stride, int32_t *counts_out,
                  int32_t *nan_bin_out, int32_t *max_b_out) {
    if (!ctx || !X || !edges_out || !counts_out || !nan_bin_out || n <= 0 || p <= 0) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    TRY(ensure_uploads(ctx));
    std::string err;
    if (gbmbin::load(ctx->bw, ctx->stager, ctx->st, X, n, p, dtype, err)) return bin_fail(ctx, err);
    if (gbmbin::edges(ctx->bw, ctx->st, n_bins, is_cat, edges_out, stride, counts_out, nan_bin_out, max_b_out, err))
        return bin_fail(ctx, err);
    return GBM_OK;
}

int gbm_upload_binned_rows(gbm_ctx *ctx, int64_t row_lo, int64_t row_hi, const double *edges, int32_t stride,
                           const int32_t *counts, const int32_t *nan_bin) {
    if (!ctx || !edges || !counts || !nan_bin) return GBM_ERR_ARG;
    int64_t n = 0;
    int p = 0;
    if (!ctx->bw || !gbmbin::shape(ctx->bw, n, p)) return fail(ctx, GBM_ERR_STATE, "call gbm_bin_edges first");
    if (row_lo < 0 || row_hi > n || row_hi <= row_lo) return fail(ctx, GBM_ERR_ARG, "bad row range");
    TRY(begin_bins(ctx, row_hi - row_lo, p, counts));
    std::string err;
    if (gbmbin::bin_blocks(ctx->bw, ctx->st, row_lo, row_hi, edges, stride, counts, nan_bin, ctx->d_xb,
                           ctx->d_bigidx, ctx->d_topbits, err))
        return bin_fail(ctx, err);
    TRY(finish_bins(ctx));
    gbmbin::release(ctx->bw);   // the keys and sort buffers are not needed after the upload
    return GBM_OK;
}

int gbm_bin_features(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype, const double *edges,
                     int32_t stride, const int32_t *counts, const int32_t *nan_bin, uint16_t *out) {
    if (!ctx || !X || !edges || !counts || !nan_bin || !out || n <= 0 || p <= 0) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    TRY(ensure_uploads(ctx));
    std::string err;
    if (gbmbin::bin_rows(ctx->bw, ctx->stager, ctx->st, X, n, p, dtype, edges, stride, counts, nan_bin, 1, out,
                         nullptr, nullptr, err))
        return bin_fail(ctx, err);
    return sync_stream(ctx);
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
    double scale = std::ldexp(1.0, ctx->S);
    k_init_grad<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_F, ctx->d_y, ctx->n, base_score, ctx->w[0], ctx->w[1],
                                                             scale, ctx->d_q);
    CKL();
    TRY(sync_stream(ctx));
    ctx->have_labels = true;
    ctx->have_targets = ctx->have_labels_mc = false;
    return GBM_OK;
}

int32_t gbm_scale_bits(const gbm_ctx *ctx) { return ctx ? ctx->S : 0; }

int gbm_get_F(gbm_ctx *ctx, double *F_out) {
    if (!ctx || !F_out) return GBM_ERR_ARG;
    if (!ctx->have_labels && !ctx->have_targets) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    CK(cudaMemcpyAsync(F_out, ctx->d_F, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st));
    return sync_stream(ctx);
}

int gbm_get_grad(gbm_ctx *ctx, double *g_out, double *h_out) {
    if (!ctx || !g_out || !h_out) return GBM_ERR_ARG;
    if (ctx->have_targets) {   // regression: the quantised gradients as the engine holds them
        CK(cudaSetDevice(ctx->dev));
        double *dg = nullptr, *dh = nullptr;
        TRY(dalloc(ctx, &dg, (size_t)ctx->n));
        int rc = dalloc(ctx, &dh, (size_t)ctx->n);
        if (rc != GBM_OK) { dfree(ctx, dg); return rc; }
        k_export_q<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_q, ctx->n, std::ldexp(1.0, -ctx->S), dg, dh);
        cudaMemcpyAsync(g_out, dg, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
        cudaMemcpyAsync(h_out, dh, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
        cudaError_t e = cudaStreamSynchronize(ctx->st);
        dfree(ctx, dg);
        dfree(ctx, dh);
        if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "gbm_get_grad: %s", cudaGetErrorString(e));
        return GBM_OK;
    }
    if (!ctx->have_labels) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    double *dg = nullptr, *dh = nullptr;
    TRY(dalloc(ctx, &dg, (size_t)ctx->n));
    int rc = dalloc(ctx, &dh, (size_t)ctx->n);
    if (rc != GBM_OK) { dfree(ctx, dg); return rc; }
    k_export_grad<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_F, ctx->d_y, ctx->n, ctx->w[0], ctx->w[1], dg, dh);
    cudaMemcpyAsync(g_out, dg, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
    cudaMemcpyAsync(h_out, dh, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
    cudaError_t e = cudaStreamSynchronize(ctx->st);
    dfree(ctx, dg);
    dfree(ctx, dh);
    if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "gbm_get_grad: %s", cudaGetErrorString(e));
    return GBM_OK;
}

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
    dfree(ctx, dg);
    dfree(ctx, dh);
    if (rc != GBM_OK) return rc;
    ctx->have_labels = false;   // the device gradients no longer follow F
    TRY(prepare_round(ctx, nfeat, P));
    std::memcpy(ctx->h_mask, inbag_mask, (size_t)ctx->n);
    CK(cudaMemcpyAsync(ctx->d_mask, ctx->h_mask, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    begin_round(ctx, 0);
    RoundFeat rf;
    TRY(setup_features(ctx, 0, feat_idx, nfeat, rf));
    TRY(enqueue_features(ctx, 0, nfeat));
    TRY(enqueue_grow(ctx, rf, P, false));
    if (device_replay(ctx, P)) {
        TRY(enqueue_replay(ctx, P));
        gbm_ctx::Slot &s = ctx->slot[0];
        CK(cudaMemcpyAsync(s.h_tout, ctx->d_tout, sizeof(TreeOut), cudaMemcpyDeviceToHost, ctx->st));
        s.h_loss[0] = 0.0;
        CK(cudaEventRecord(s.done, ctx->st));
        TRY(wait_slot(ctx, 0));
        return harvest(ctx, 0, nfeat, P, out, nullptr);
    }
    HostTree T;
    TRY(replay_on_host(ctx, rf, P, T));
    write_tree(T, tree_need(P), out);
    return GBM_OK;
}

// One round from the staged in-bag mask (on the device) and feature list:
// growth, the tree (device replay, or host replay for capped levels), the F
// update, the loss, and the wait for all of it.
static int round_body(gbm_ctx *ctx, int si, const int32_t *feat_idx, int32_t nfeat, const gbm_params *P,
                      gbm_tree_out *out, double *train_loss, bool compacted) {
    gbm_ctx::Slot &s = ctx->slot[si];
    RoundFeat rf;
    TRY(setup_features(ctx, si, feat_idx, nfeat, rf));
    TRY(enqueue_features(ctx, si, nfeat));
    TRY(enqueue_grow(ctx, rf, P, compacted));
    const bool dev = device_replay(ctx, P);
    HostTree T;
    if (dev) {
        TRY(enqueue_replay(ctx, P));
        CK(cudaMemcpyAsync(s.h_tout, ctx->d_tout, sizeof(TreeOut), cudaMemcpyDeviceToHost, ctx->st));
    } else {
        TRY(replay_on_host(ctx, rf, P, T));
        if (T.nc > 256) return fail(ctx, GBM_ERR_UNSUPPORTED, "tree with %d nodes exceeds 256", T.nc);
        TreeDev td;
        std::memset(&td, 0, sizeof td);
        td.n = T.nc;
        for (int k = 0; k < T.nc; k++) {
            td.feat[k] = T.tf[k];
            td.thr[k] = dev_thr(T.tt[k] & 0xffffffffll, (int)(T.tt[k] >> 32));
            td.left[k] = T.tl[k];
            td.right[k] = T.tr[k];
            td.val[k] = T.tv[k];
        }
        CK(cudaMemcpyAsync(ctx->d_tree, &td, sizeof td, cudaMemcpyHostToDevice, ctx->st));
    }
    TRY(enqueue_update(ctx, P, out->leaf_of_row != nullptr, s.h_loss));
    if (out->leaf_of_row)
        CK(cudaMemcpyAsync(out->leaf_of_row, ctx->d_leaf, sizeof(int32_t) * ctx->n, cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaEventRecord(s.done, ctx->st));
    TRY(wait_slot(ctx, si));
    if (dev) return harvest(ctx, si, nfeat, P, out, train_loss);
    TRY(p2p_check(ctx, si));
    if (ctx->profiling) TRY(collect_slot_timing(ctx, si));
    if (train_loss) *train_loss = -s.h_loss[0] / (double)ctx->n_global;
    write_tree(T, tree_need(P), out);
    return GBM_OK;
}

// ---- regression (E:2607-2705) ------------------------------------------------

// S for the next round from the largest |g| (every rank's: each proposes its
// S, the all-reduce of a one-hot table gives the smallest), then the
// quantised gradients.
static int reg_requantize(gbm_ctx *ctx, double gmax) {
    int S = scale_bits_for(ctx->reg_mae ? 1.0 : gmax);
    if (ctx->comm) {
        long long tab[128] = {};
        const int slot = std::min(127, std::max(0, S + 64));
        tab[slot] = 1;
        CK(cudaMemcpyAsync(ctx->d_stab, tab, sizeof tab, cudaMemcpyHostToDevice, ctx->st));
        TRY(allreduce_i64(ctx, ctx->d_stab, 128));
        CK(cudaMemcpyAsync(tab, ctx->d_stab, sizeof tab, cudaMemcpyDeviceToHost, ctx->st));
        TRY(sync_stream(ctx));
        for (int k = 0; k < 128; k++)
            if (tab[k]) { S = k - 64; break; }
    }
    ctx->S = S;
    k_reg_quant<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_F, ctx->d_yr, ctx->n, ctx->reg_mae,
                                                            std::ldexp(1.0, S), ctx->d_q);
    CKL();
    return GBM_OK;
}

int gbm_upload_targets(gbm_ctx *ctx, const double *y, double init_score, int32_t loss, int64_t n_global) {
    if (!ctx || !y || (loss != 0 && loss != 1) || !std::isfinite(init_score)) return GBM_ERR_ARG;
    if (!ctx->have_bins) return fail(ctx, GBM_ERR_STATE, "upload bins before targets");
    double gmax = 0.0;
    for (int64_t i = 0; i < ctx->n; i++) {
        if (!std::isfinite(y[i])) return fail(ctx, GBM_ERR_ARG, "target %lld is not finite", (long long)i);
        gmax = std::max(gmax, std::fabs(init_score - y[i]));
    }
    CK(cudaSetDevice(ctx->dev));
    ctx->reg_mae = loss;
    ctx->base = init_score;
    ctx->n_global = n_global > 0 ? n_global : ctx->n;
    TRY(dalloc(ctx, &ctx->d_yr, (size_t)ctx->n));
    TRY(dalloc(ctx, &ctx->d_gmax_part, (size_t)ctx->upd_blocks));
    TRY(dalloc(ctx, &ctx->d_gmax, 1));
    TRY(dalloc(ctx, &ctx->d_stab, 128));
    CK(cudaMemcpyAsync(ctx->d_yr, y, sizeof(double) * (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    k_fill<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_F, ctx->n, init_score);
    CKL();
    TRY(reg_requantize(ctx, gmax));
    TRY(sync_stream(ctx));
    ctx->have_labels = ctx->have_labels_mc = false;
    ctx->have_targets = true;
    return GBM_OK;
}

// One regression round on slot si (begun by the caller), its in-bag mask in
// d_mask (and, with `compacted`, its root row list in d_rows).
static int round_reg_body(gbm_ctx *ctx, int si, const int32_t *feat_idx, int32_t nfeat, const gbm_params *P,
                          gbm_tree_out *out, double *train_loss, bool compacted) {
    gbm_ctx::Slot &s = ctx->slot[si];
    RoundFeat rf;
    TRY(setup_features(ctx, si, feat_idx, nfeat, rf));
    TRY(enqueue_features(ctx, si, nfeat));
    TRY(enqueue_grow(ctx, rf, P, compacted));
    if (device_replay(ctx, P)) {
        TRY(enqueue_replay(ctx, P));
        CK(cudaMemcpyAsync(s.h_tout, ctx->d_tout, sizeof(TreeOut), cudaMemcpyDeviceToHost, ctx->st));
        CK(cudaEventRecord(s.done, ctx->st));
        TRY(wait_slot(ctx, si));
        TRY(harvest(ctx, si, nfeat, P, out, nullptr));
    } else {
        HostTree T;
        TRY(replay_on_host(ctx, rf, P, T));
        if (T.nc > 256) return fail(ctx, GBM_ERR_UNSUPPORTED, "tree with %d nodes exceeds 256", T.nc);
        TreeDev td;
        std::memset(&td, 0, sizeof td);
        td.n = T.nc;
        for (int j = 0; j < T.nc; j++) {
            td.feat[j] = T.tf[j];
            td.thr[j] = dev_thr(T.tt[j] & 0xffffffffll, (int)(T.tt[j] >> 32));
            td.left[j] = T.tl[j];
            td.right[j] = T.tr[j];
            td.val[j] = T.tv[j];
        }
        CK(cudaMemcpyAsync(ctx->d_tree, &td, sizeof td, cudaMemcpyHostToDevice, ctx->st));
        TRY(sync_stream(ctx));
        write_tree(T, tree_need(P), out);
    }
    TRY(launch(ctx, k_update_reg, dim3(ctx->upd_blocks), dim3(kUpdThreads), 0, ctx->st, (const TreeDev *)ctx->d_tree,
               (const uint8_t *)ctx->d_xb, ctx->n, P->learning_rate, ctx->d_F, (const double *)ctx->d_yr,
               ctx->reg_mae, out->leaf_of_row ? ctx->d_leaf : (int32_t *)nullptr, ctx->d_loss_part,
               ctx->d_gmax_part, (const int32_t *)ctx->d_bigidx, (const uint32_t *)ctx->d_topbits));
    TRY(launch(ctx, k_sum_partials, dim3(1), dim3(256), 0, ctx->st, ctx->d_loss_part, ctx->upd_blocks, ctx->d_loss));
    TRY(launch(ctx, k_max_partials, dim3(1), dim3(32), 0, ctx->st, (const double *)ctx->d_gmax_part,
               ctx->upd_blocks, ctx->d_gmax));
    if (ctx->comm) TRY(allreduce_f64(ctx, ctx->d_loss, 1));
    if (out->leaf_of_row)
        CK(cudaMemcpyAsync(out->leaf_of_row, ctx->d_leaf, sizeof(int32_t) * ctx->n, cudaMemcpyDeviceToHost, ctx->st));
    double gmax = 0.0;
    CK(cudaMemcpyAsync(s.h_loss, ctx->d_loss, sizeof(double), cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaMemcpyAsync(&gmax, ctx->d_gmax, sizeof(double), cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    if (train_loss) *train_loss = s.h_loss[0] / (double)ctx->n_global;
    TRY(reg_requantize(ctx, gmax));   // the next round's gradients
    return sync_stream(ctx);
}

int gbm_round_reg(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
                  const gbm_params *P, gbm_tree_out *out, double *train_loss) {
    if (!ctx || !inbag_mask || !feat_idx || !P || !out) return GBM_ERR_ARG;
    if (!ctx->have_targets) return fail(ctx, GBM_ERR_STATE, "upload bins and gbm_upload_targets first");
    TRY(check_tree_args(ctx, nfeat, P, out));
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nfeat, P));
    std::memcpy(ctx->h_mask, inbag_mask, (size_t)ctx->n);
    CK(cudaMemcpyAsync(ctx->d_mask, ctx->h_mask, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    begin_round(ctx, 0);
    return round_reg_body(ctx, 0, feat_idx, nfeat, P, out, train_loss, false);
}

int gbm_round_reg_sampled(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *P,
                          gbm_tree_out *out, double *train_loss) {
    if (!ctx || !sampler || !P || !out || row_offset < 0) return GBM_ERR_ARG;
    if (!ctx->have_targets) return fail(ctx, GBM_ERR_STATE, "upload bins and gbm_upload_targets first");
    const int32_t nf = gbm_sampler_n_feat(sampler);
    TRY(check_tree_args(ctx, nf, P, out));
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nf, P));
    const int si = (int)(gbm_sampler_taken(sampler) % gbm_ctx::kRing);
    begin_round(ctx, si);
    TRY(take_sample(ctx, si, sampler, row_offset));
    TRY(enqueue_sample(ctx, si, gbm_sampler_rows(sampler), gbm_sampler_n_sub(sampler),
                       gbm_sampler_shuffles_rows(sampler) != 0, row_offset, 0, dev_rows_of(sampler)));
    TRY(wait_copied(ctx, ctx->slot[si]));
    return round_reg_body(ctx, si, ctx->feat_buf.data(), nf, P, out, train_loss, true);
}

// ---- multi-class softmax (E:2949-3065) ---------------------------------------

int gbm_upload_labels_mc(gbm_ctx *ctx, const uint8_t *y, int32_t n_classes, const double *class_w,
                         int64_t n_global) {
    if (!ctx || !y || !class_w || n_classes < 3 || n_classes > kMaxClasses) return GBM_ERR_ARG;
    if (!ctx->have_bins) return fail(ctx, GBM_ERR_STATE, "upload bins before labels");
    double wmax = 0.0;
    for (int k = 0; k < n_classes; k++) {
        if (!(class_w[k] > 0.0) || !std::isfinite(class_w[k]))
            return fail(ctx, GBM_ERR_ARG, "class weights must be finite and > 0");
        wmax = std::max(wmax, class_w[k]);
    }
    for (int64_t i = 0; i < ctx->n; i++)
        if (y[i] >= n_classes) return fail(ctx, GBM_ERR_ARG, "label %d of row %lld >= %d classes", (int)y[i], (long long)i,
                                           n_classes);
    CK(cudaSetDevice(ctx->dev));
    ctx->K = n_classes;
    ctx->n_global = n_global > 0 ? n_global : ctx->n;
    // |g| <= w and h <= w/4 for every class, as in the binary case
    ctx->S = scale_bits_for(wmax);
    TRY(dalloc(ctx, &ctx->d_Fmc, (size_t)ctx->n * n_classes));
    TRY(dalloc(ctx, &ctx->d_qmc, (size_t)ctx->n * n_classes));
    TRY(dalloc(ctx, &ctx->d_wmc, (size_t)n_classes));
    CK(cudaMemsetAsync(ctx->d_Fmc, 0, sizeof(double) * (size_t)ctx->n * n_classes, ctx->st));   // F starts at 0 (E:2959)
    CK(cudaMemcpyAsync(ctx->d_wmc, class_w, sizeof(double) * n_classes, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->d_y, y, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    k_softmax_grad<<<ctx->upd_blocks, kUpdThreads, 0, ctx->st>>>(ctx->d_Fmc, ctx->d_y, ctx->n, n_classes, ctx->d_wmc,
                                                                 std::ldexp(1.0, ctx->S), ctx->d_qmc, ctx->d_loss_part);
    CKL();
    TRY(sync_stream(ctx));
    ctx->have_labels = ctx->have_targets = false;   // the other objectives' state no longer follows
    ctx->have_labels_mc = true;
    return GBM_OK;
}

// One multi-class round on slot si, its in-bag mask in d_mask (and, with
// `compacted`, its root row list in d_rows).
static int round_mc_body(gbm_ctx *ctx, int si, const int32_t *feat_idx, int32_t nfeat, const gbm_params *P,
                         gbm_tree_out *outs, double *train_loss, bool compacted) {
    const int K = ctx->K;
    longlong2 *const q_bin = ctx->d_q;
    int rc = GBM_OK;
    bool want_leaf = false;
    for (int k = 0; k < K; k++) want_leaf |= outs[k].leaf_of_row != nullptr;
    // K trees on the same sample and features, each from its class's
    // gradients of the round's start (E:2995-3006).  With the tree replayed
    // on the device and no per-row leaves asked for, the K trees and class
    // updates are queued back to back (each tree's record copied to its own
    // pinned slot) and the host waits once, after the round's gradients.
    const bool batched = device_replay(ctx, P) && !want_leaf;
    if (batched) {
        TRY(halloc(ctx, &ctx->h_tout_mc, (size_t)K));
        RoundFeat rf;   // (the caller began slot si's round)
        TRY(setup_features(ctx, si, feat_idx, nfeat, rf));
        TRY(enqueue_features(ctx, si, nfeat));
        for (int k = 0; k < K && rc == GBM_OK; k++) {
            ctx->d_q = ctx->d_qmc + (int64_t)k * ctx->n;
            // the row list from the mask, per tree (a partition overwrites it)
            rc = enqueue_grow(ctx, rf, P, compacted && k == 0);
            if (rc == GBM_OK) rc = enqueue_replay(ctx, P);
            if (rc == GBM_OK && cudaMemcpyAsync(&ctx->h_tout_mc[k], ctx->d_tout, sizeof(TreeOut),
                                                cudaMemcpyDeviceToHost, ctx->st) != cudaSuccess)
                rc = fail(ctx, GBM_ERR_CUDA, "tree copy");
            if (rc == GBM_OK)
                rc = launch(ctx, k_update_class, dim3(ctx->upd_blocks), dim3(kUpdThreads), 0, ctx->st,
                            (const TreeDev *)ctx->d_tree, (const uint8_t *)ctx->d_xb, ctx->n, P->learning_rate,
                            ctx->d_Fmc + (int64_t)k * ctx->n, (int32_t *)nullptr, (const int32_t *)ctx->d_bigidx,
                            (const uint32_t *)ctx->d_topbits);
        }
    }
    for (int k = 0; k < K && rc == GBM_OK && !batched; k++) {
        ctx->d_q = ctx->d_qmc + (int64_t)k * ctx->n;
        gbm_ctx::Slot &s = ctx->slot[si];
        begin_round(ctx, si);
        RoundFeat rf;
        rc = setup_features(ctx, si, feat_idx, nfeat, rf);
        if (rc == GBM_OK) rc = enqueue_features(ctx, si, nfeat);
        if (rc == GBM_OK) rc = enqueue_grow(ctx, rf, P, compacted && k == 0);   // the row list, per tree
        if (rc != GBM_OK) break;
        if (device_replay(ctx, P)) {
            rc = enqueue_replay(ctx, P);
            if (rc == GBM_OK && cudaMemcpyAsync(s.h_tout, ctx->d_tout, sizeof(TreeOut), cudaMemcpyDeviceToHost,
                                                ctx->st) != cudaSuccess)
                rc = fail(ctx, GBM_ERR_CUDA, "tree copy");
            if (rc == GBM_OK && cudaEventRecord(s.done, ctx->st) != cudaSuccess) rc = fail(ctx, GBM_ERR_CUDA, "event");
            if (rc == GBM_OK) rc = wait_slot(ctx, si);
            if (rc == GBM_OK) rc = harvest(ctx, si, nfeat, P, &outs[k], nullptr);
        } else {
            HostTree T;
            rc = replay_on_host(ctx, rf, P, T);
            if (rc == GBM_OK && T.nc > 256) rc = fail(ctx, GBM_ERR_UNSUPPORTED, "tree with %d nodes exceeds 256", T.nc);
            if (rc == GBM_OK) {
                TreeDev td;
                std::memset(&td, 0, sizeof td);
                td.n = T.nc;
                for (int j = 0; j < T.nc; j++) {
                    td.feat[j] = T.tf[j];
                    td.thr[j] = dev_thr(T.tt[j] & 0xffffffffll, (int)(T.tt[j] >> 32));
                    td.left[j] = T.tl[j];
                    td.right[j] = T.tr[j];
                    td.val[j] = T.tv[j];
                }
                if (cudaMemcpyAsync(ctx->d_tree, &td, sizeof td, cudaMemcpyHostToDevice, ctx->st) != cudaSuccess ||
                    cudaStreamSynchronize(ctx->st) != cudaSuccess)
                    rc = fail(ctx, GBM_ERR_CUDA, "tree upload");
                write_tree(T, tree_need(P), &outs[k]);
            }
        }
        if (rc == GBM_OK)
            rc = launch(ctx, k_update_class, dim3(ctx->upd_blocks), dim3(kUpdThreads), 0, ctx->st,
                        (const TreeDev *)ctx->d_tree, (const uint8_t *)ctx->d_xb, ctx->n, P->learning_rate,
                        ctx->d_Fmc + (int64_t)k * ctx->n,
                        outs[k].leaf_of_row ? ctx->d_leaf : (int32_t *)nullptr, (const int32_t *)ctx->d_bigidx,
                        (const uint32_t *)ctx->d_topbits);
        if (rc == GBM_OK && outs[k].leaf_of_row &&
            (cudaMemcpyAsync(outs[k].leaf_of_row, ctx->d_leaf, sizeof(int32_t) * ctx->n, cudaMemcpyDeviceToHost,
                             ctx->st) != cudaSuccess || cudaStreamSynchronize(ctx->st) != cudaSuccess))
            rc = fail(ctx, GBM_ERR_CUDA, "leaf copy");
    }
    ctx->d_q = q_bin;
    TRY(rc);
    // the next round's gradients of every class and this round's loss (E:3008)
    TRY(launch(ctx, k_softmax_grad, dim3(ctx->upd_blocks), dim3(kUpdThreads), 0, ctx->st, (const double *)ctx->d_Fmc,
               (const uint8_t *)ctx->d_y, ctx->n, K, (const double *)ctx->d_wmc, std::ldexp(1.0, ctx->S), ctx->d_qmc,
               ctx->d_loss_part));
    TRY(launch(ctx, k_sum_partials, dim3(1), dim3(256), 0, ctx->st, ctx->d_loss_part, ctx->upd_blocks, ctx->d_loss));
    if (ctx->comm) TRY(allreduce_f64(ctx, ctx->d_loss, 1));
    double loss = 0.0;
    CK(cudaMemcpyAsync(ctx->slot[si].h_loss, ctx->d_loss, sizeof(double), cudaMemcpyDeviceToHost, ctx->st));
    TRY(sync_stream(ctx));
    if (batched) {
        if (ctx->profiling) TRY(collect_slot_timing(ctx, si));
        TRY(p2p_check(ctx, si));
        for (int k = 0; k < K; k++)
            TRY(take_tree(ctx, ctx->h_tout_mc[k], ctx->slot[si].upd_per_row, nfeat, P, &outs[k]));
    }
    loss = ctx->slot[si].h_loss[0];
    if (train_loss) *train_loss = -loss / (double)ctx->n_global;
    return GBM_OK;
}


int gbm_round_mc(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
                 const gbm_params *P, gbm_tree_out *outs, double *train_loss) {
    if (!ctx || !inbag_mask || !feat_idx || !P || !outs) return GBM_ERR_ARG;
    if (!ctx->have_labels_mc) return fail(ctx, GBM_ERR_STATE, "upload bins and gbm_upload_labels_mc first");
    for (int k = 0; k < ctx->K; k++) TRY(check_tree_args(ctx, nfeat, P, &outs[k]));
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nfeat, P));
    std::memcpy(ctx->h_mask, inbag_mask, (size_t)ctx->n);
    CK(cudaMemcpyAsync(ctx->d_mask, ctx->h_mask, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    begin_round(ctx, 0);
    return round_mc_body(ctx, 0, feat_idx, nfeat, P, outs, train_loss, false);
}

int gbm_round_mc_sampled(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *P,
                         gbm_tree_out *outs, double *train_loss) {
    if (!ctx || !sampler || !P || !outs || row_offset < 0) return GBM_ERR_ARG;
    if (!ctx->have_labels_mc) return fail(ctx, GBM_ERR_STATE, "upload bins and gbm_upload_labels_mc first");
    const int32_t nf = gbm_sampler_n_feat(sampler);
    for (int k = 0; k < ctx->K; k++) TRY(check_tree_args(ctx, nf, P, &outs[k]));
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nf, P));
    const int si = (int)(gbm_sampler_taken(sampler) % gbm_ctx::kRing);
    begin_round(ctx, si);
    TRY(take_sample(ctx, si, sampler, row_offset));
    TRY(enqueue_sample(ctx, si, gbm_sampler_rows(sampler), gbm_sampler_n_sub(sampler),
                       gbm_sampler_shuffles_rows(sampler) != 0, row_offset, 0, dev_rows_of(sampler)));
    TRY(wait_copied(ctx, ctx->slot[si]));
    return round_mc_body(ctx, si, ctx->feat_buf.data(), nf, P, outs, train_loss, true);
}

int gbm_get_F_mc(gbm_ctx *ctx, double *F_out) {
    if (!ctx || !F_out) return GBM_ERR_ARG;
    if (!ctx->have_labels_mc) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    CK(cudaMemcpyAsync(F_out, ctx->d_Fmc, sizeof(double) * (size_t)ctx->n * ctx->K, cudaMemcpyDeviceToHost, ctx->st));
    return sync_stream(ctx);
}

int gbm_get_grad_mc(gbm_ctx *ctx, int32_t k, double *g_out, double *h_out) {
    if (!ctx || !g_out || !h_out) return GBM_ERR_ARG;
    if (!ctx->have_labels_mc || k < 0 || k >= ctx->K) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    double *dg = nullptr, *dh = nullptr;
    TRY(dalloc(ctx, &dg, (size_t)ctx->n));
    int rc = dalloc(ctx, &dh, (size_t)ctx->n);
    if (rc != GBM_OK) { dfree(ctx, dg); return rc; }
    k_export_q<<<grid_for(ctx->n, 256), 256, 0, ctx->st>>>(ctx->d_qmc + (int64_t)k * ctx->n, ctx->n,
                                                           std::ldexp(1.0, -ctx->S), dg, dh);
    cudaMemcpyAsync(g_out, dg, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
    cudaMemcpyAsync(h_out, dh, sizeof(double) * ctx->n, cudaMemcpyDeviceToHost, ctx->st);
    cudaError_t e = cudaStreamSynchronize(ctx->st);
    dfree(ctx, dg);
    dfree(ctx, dh);
    if (e != cudaSuccess) return fail(ctx, GBM_ERR_CUDA, "gbm_get_grad_mc: %s", cudaGetErrorString(e));
    return GBM_OK;
}

int gbm_round(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
              const gbm_params *P, gbm_tree_out *out, double *train_loss) {
    if (!ctx || !inbag_mask || !feat_idx || !P || !out) return GBM_ERR_ARG;
    if (!ctx->have_labels) return fail(ctx, GBM_ERR_STATE, "upload bins and labels before gbm_round");
    TRY(check_tree_args(ctx, nfeat, P, out));
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nfeat, P));
    std::memcpy(ctx->h_mask, inbag_mask, (size_t)ctx->n);
    CK(cudaMemcpyAsync(ctx->d_mask, ctx->h_mask, (size_t)ctx->n, cudaMemcpyHostToDevice, ctx->st));
    begin_round(ctx, 0);
    return round_body(ctx, 0, feat_idx, nfeat, P, out, train_loss, false);
}

int gbm_round_sampled(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *P,
                      gbm_tree_out *out, double *train_loss) {
    if (!ctx || !sampler || !P || !out || row_offset < 0) return GBM_ERR_ARG;
    if (!ctx->have_labels) return fail(ctx, GBM_ERR_STATE, "upload bins and labels before gbm_round_sampled");
    int32_t nf = gbm_sampler_n_feat(sampler);
    TRY(check_tree_args(ctx, nf, P, out));
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nf, P));
    const int si = (int)(gbm_sampler_taken(sampler) % gbm_ctx::kRing);
    begin_round(ctx, si);
    TRY(take_sample(ctx, si, sampler, row_offset));
    TRY(enqueue_sample(ctx, si, gbm_sampler_rows(sampler), gbm_sampler_n_sub(sampler),
                       gbm_sampler_shuffles_rows(sampler) != 0, row_offset, 0, dev_rows_of(sampler)));
    TRY(wait_ev(ctx, ctx->st, ctx->slot[si].copied));
    return round_body(ctx, si, ctx->feat_buf.data(), nf, P, out, train_loss, true);
}

int gbm_fit_rounds(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *P, int32_t n_rounds,
                   gbm_tree_out *outs, double *train_loss) {
    if (!ctx || !sampler || !P || !outs || !train_loss || row_offset < 0 || n_rounds < 0) return GBM_ERR_ARG;
    if (!ctx->have_labels) return fail(ctx, GBM_ERR_STATE, "upload bins and labels before gbm_fit_rounds");
    int32_t nf = gbm_sampler_n_feat(sampler);
    bool leaf = false;
    for (int r = 0; r < n_rounds; r++) {
        TRY(check_tree_args(ctx, nf, P, &outs[r]));
        leaf |= outs[r].leaf_of_row != nullptr;
    }
    CK(cudaSetDevice(ctx->dev));
    TRY(prepare_round(ctx, nf, P));
    if (leaf || !device_replay(ctx, P)) {
        for (int r = 0; r < n_rounds; r++)
            TRY(gbm_round_sampled(ctx, sampler, row_offset, P, &outs[r], &train_loss[r]));
        return GBM_OK;
    }
    const int R = gbm_ctx::kRing;
    const int64_t N = gbm_sampler_rows(sampler), m = gbm_sampler_n_sub(sampler);
    const bool rows_on = gbm_sampler_shuffles_rows(sampler) != 0;
    const DevRows dr = dev_rows_of(sampler);
    if (rows_on) TRY(ensure_shuffle(ctx, N));   // before any capture: no allocation inside one
    // With several ranks a round is replayed from graphs: each round's ~13
    // collective enqueues cost the host more than the GPU needs for the
    // round.  One GPU launches eagerly (programmatic dependent launch
    // already hides the gaps there, and capturing costs a first fit time).
    const bool graphs = ctx->comm != nullptr;
    if (graphs) {
        const std::string key = graph_key(ctx, P, nf, N, m, rows_on, row_offset) + (dr.on ? "/dev" : "");
        if (key != ctx->graph_key) {
            drop_graphs(ctx);
            for (int si = 0; si < R; si++) TRY(capture_round(ctx, si, nf, P, N, m, rows_on, row_offset, dr));
            ctx->graph_key = key;
        }
    }
    const int64_t r0 = gbm_sampler_taken(sampler);
    for (int k = 0; k < n_rounds + R; k++) {
        const int si = (int)((r0 + k) % R);
        if (k >= R) {
            TRY(wait_slot(ctx, si));
            TRY(harvest(ctx, si, nf, P, &outs[k - R], &train_loss[k - R]));
        }
        if (k >= n_rounds) continue;
        gbm_ctx::Slot &s = ctx->slot[si];
        if (!graphs) {
            begin_round(ctx, si);
            TRY(take_sample(ctx, si, sampler, row_offset));
            RoundFeat rf;
            TRY(setup_features(ctx, si, ctx->feat_buf.data(), nf, rf));   // before the sample packs its features
            TRY(enqueue_sample(ctx, si, N, m, rows_on, row_offset, nf, dr));
            TRY(wait_copied(ctx, s));
            TRY(enqueue_features(ctx, si, nf));
            TRY(enqueue_grow(ctx, rf, P, true));
            TRY(enqueue_replay(ctx, P));
            TRY(enqueue_update(ctx, P, false, s.h_loss));
            CK(cudaMemcpyAsync(s.h_tout, ctx->d_tout, sizeof(TreeOut), cudaMemcpyDeviceToHost, ctx->st));
            CK(cudaEventRecord(s.done, ctx->st));
            continue;
        }
        ctx->cur_slot = si;
        TRY(take_sample(ctx, si, sampler, row_offset));
        RoundFeat rf;
        TRY(setup_features(ctx, si, ctx->feat_buf.data(), nf, rf));
        s.tused = s.g_tpairs;
        s.tdone = 0;
        CK(cudaGraphLaunch(s.g_cst, ctx->cst));
        CK(cudaGraphLaunch(s.g_st, ctx->st));
        ctx->launches += s.g_launches;
        ctx->hist_launches += s.g_hist;
        ctx->waves += s.g_waves;
        ctx->comm_bytes += s.g_comm_bytes;
    }
    return GBM_OK;
}

// ---- failure detection self test ----------------------------------------------

int gbm_test_peer_wait(int32_t device, int32_t timeout_ms) {
    if (timeout_ms <= 0 || timeout_ms > 10000) return GBM_ERR_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return GBM_ERR_CUDA;
    const int N = 2, nf = 1;
    const int64_t words = slot_words_for(nf);
    long long *pst = nullptr, *out = nullptr, **peers = nullptr;
    unsigned long long *sync = nullptr;
    int rc = GBM_OK;
    if (cudaMalloc(&pst, sizeof(long long) * (size_t)(2 * words)) != cudaSuccess ||
        cudaMalloc(&out, sizeof(long long) * (size_t)words) != cudaSuccess ||
        cudaMalloc(&peers, sizeof(long long *) * N) != cudaSuccess ||
        cudaMalloc(&sync, sizeof(unsigned long long) * (N + kSyncLocal)) != cudaSuccess)
        rc = GBM_ERR_ALLOC;
    if (rc == GBM_OK) {
        // rank 0 of 2 has signalled one level; rank 1 never will
        std::vector<unsigned long long> s0((size_t)(N + kSyncLocal), 0ull);
        s0[(size_t)(N + kSyncSent)] = 1;
        long long *pp[2] = {pst, pst};
        unsigned long long err = 0;
        if (cudaMemset(pst, 0, sizeof(long long) * (size_t)(2 * words)) != cudaSuccess ||
            cudaMemcpy(sync, s0.data(), sizeof(unsigned long long) * s0.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(peers, pp, sizeof pp, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = GBM_ERR_CUDA;
        } else {
            k_peer_sum<<<1, 256>>>(peers, words, sync, 0, N, nullptr, nf, out, pst, (long long)timeout_ms * 1000000ll);
            if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
                cudaMemcpy(&err, sync + N + kSyncErr, sizeof err, cudaMemcpyDeviceToHost) != cudaSuccess)
                rc = GBM_ERR_CUDA;
            else
                rc = err ? GBM_ERR_TIMEOUT : GBM_OK;
        }
    }
    void *ptrs[] = {pst, out, peers, sync};
    for (void *q : ptrs) if (q) cudaFree(q);
    return rc;
}

// ---- predict ------------------------------------------------------------------

int gbm_check_model(const gbm_packed *m, int32_t n_features, char *errbuf, int32_t errlen) {
    if (!m || m->n_trees < 0 || !m->offsets || n_features <= 0) {
        if (errbuf && errlen > 0) snprintf(errbuf, (size_t)errlen, "null model or empty size");
        return GBM_ERR_ARG;
    }
    std::vector<PNode> nodes;
    std::vector<double> vals;
    std::string err;
    int rc = pack_model(err, m, n_features, nodes, vals);
    if (rc && errbuf && errlen > 0) snprintf(errbuf, (size_t)errlen, "%s", err.c_str());
    return rc;
}

int gbm_predict_set_model(gbm_ctx *ctx, const gbm_packed *m, int32_t n_features) {
    if (!ctx || !m || m->n_trees < 0 || !m->offsets || n_features <= 0) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    int32_t T = m->n_trees;
    std::vector<PNode> nodes;
    std::vector<double> vals;
    std::vector<uint32_t> n32;
    std::vector<double> v32;
    std::vector<int32_t> dep;
    std::string err;
    bool has_nr = false;
    if (int rc = pack_model(err, m, n_features, nodes, vals, &n32, &v32, &dep, &has_nr))
        return fail(ctx, rc, "%s", err.c_str());
    CK(cudaSetDevice(ctx->dev));
    int64_t total = (int64_t)nodes.size();
    if (total > ctx->p_nodes_cap) {
        TRY(dalloc(ctx, &ctx->d_pnodes, (size_t)total * sizeof(PNode)));
        TRY(dalloc(ctx, &ctx->d_pvals, (size_t)total));
        ctx->p_nodes_cap = total;
    }
    if (T + 1 > ctx->p_trees_cap) {
        TRY(dalloc(ctx, &ctx->d_poff, (size_t)T + 1));
        TRY(dalloc(ctx, &ctx->d_pchunk, (size_t)T + 2));   // the count sits in the last int4
        TRY(dalloc(ctx, &ctx->d_pdep, (size_t)T + 1));
        ctx->p_trees_cap = T + 1;
    }
    ctx->p_packed = !n32.empty();
    ctx->p_packed_nr = has_nr;
    if (ctx->p_packed) {
        CK(cudaMemcpyAsync(ctx->d_pnodes, n32.data(), sizeof(uint32_t) * total, cudaMemcpyHostToDevice, ctx->st));
        CK(cudaMemcpyAsync(ctx->d_pvals, v32.data(), sizeof(double) * total, cudaMemcpyHostToDevice, ctx->st));
        if (T > 0)
            CK(cudaMemcpyAsync(ctx->d_pdep, dep.data(), sizeof(int32_t) * T, cudaMemcpyHostToDevice, ctx->st));
    } else {
        CK(cudaMemcpyAsync(ctx->d_pnodes, nodes.data(), sizeof(PNode) * total, cudaMemcpyHostToDevice, ctx->st));
        CK(cudaMemcpyAsync(ctx->d_pvals, vals.data(), sizeof(double) * total, cudaMemcpyHostToDevice, ctx->st));
    }
    CK(cudaMemcpyAsync(ctx->d_poff, m->offsets, sizeof(int32_t) * (T + 1), cudaMemcpyHostToDevice, ctx->st));
    // the ensemble's chunks of whole trees, cut once per model on the device
    k_pred_chunks<<<1, 32, 0, ctx->st>>>(ctx->d_poff, T, ctx->d_pchunk,
                                         reinterpret_cast<int32_t *>(ctx->d_pchunk + T + 1));
    CKL();
    ctx->p_ntree = T;
    ctx->p_nfeat = n_features;
    return sync_stream(ctx);
}

static int predict_alloc(gbm_ctx *ctx, int64_t n, int32_t p) {
    if (ctx->dev < 0) return GBM_ERR_STATE;
    if (ctx->p_nfeat && p != ctx->p_nfeat) return fail(ctx, GBM_ERR_ARG, "X has %d features, model %d", p, ctx->p_nfeat);
    CK(cudaSetDevice(ctx->dev));
    if (n * p > ctx->pn_cap) {
        TRY(dalloc(ctx, &ctx->d_px, (size_t)(n * p)));
        ctx->pn_cap = n * p;
    }
    TRY(dalloc(ctx, &ctx->d_pF, (size_t)n));
    TRY(dalloc(ctx, &ctx->d_pP, (size_t)n));
    TRY(ensure_uploads(ctx));
    ctx->pn = n;
    ctx->pp = p;
    ctx->p_top = false;
    return GBM_OK;
}

// The predict rows' top-bit state for the features flagged in bigidx [p]
// (-1: not a 257-bin feature): zeroed bits, ready for the binning to set.
static int predict_top_alloc(gbm_ctx *ctx, const std::vector<int32_t> &bigidx, int nbig) {
    ctx->p_top = nbig > 0;
    if (!nbig) return GBM_OK;
    const size_t words = (size_t)nbig * (size_t)((ctx->pn + 31) >> 5);
    TRY(dalloc(ctx, &ctx->d_pbigidx, (size_t)ctx->pp));
    TRY(dalloc(ctx, &ctx->d_ptopbits, words));
    CK(cudaMemcpyAsync(ctx->d_pbigidx, bigidx.data(), sizeof(int32_t) * ctx->pp, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemsetAsync(ctx->d_ptopbits, 0, sizeof(uint32_t) * words, ctx->st));
    return sync_stream(ctx);   // bigidx is host memory of the caller's frame
}

int gbm_predict_upload(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p) {
    if (!ctx || !xbin || n <= 0 || p <= 0) return GBM_ERR_ARG;
    TRY(predict_alloc(ctx, n, p));
    uint8_t *px = ctx->d_px;
    auto dst = [px, p](int64_t r0, int64_t) { return static_cast<void *>(px + r0 * p); };
    std::string err;
    if (gbmh2d::stream_rows(ctx->stager, ctx->st, xbin, n, (size_t)p, gbmh2d::Pack::Copy, 0, dst, nullptr, err))
        return fail(ctx, GBM_ERR_CUDA, "predict upload: %s", err.c_str());
    return GBM_OK;
}

int gbm_predict_upload_u16(gbm_ctx *ctx, const uint16_t *xbin, int64_t n, int32_t p) {
    if (!ctx || !xbin || n <= 0 || p <= 0) return GBM_ERR_ARG;
    TRY(predict_alloc(ctx, n, p));
    uint8_t *px = ctx->d_px;
    auto dst = [px, p](int64_t r0, int64_t) { return static_cast<void *>(px + r0 * p); };
    std::string err;
    std::vector<int64_t> wide;   // ids above 255, read as bin 256
    if (gbmh2d::stream_rows(ctx->stager, ctx->st, xbin, n, 2 * (size_t)p, gbmh2d::Pack::U16toU8, 0, dst, nullptr,
                            err, &wide))
        return fail(ctx, GBM_ERR_CUDA, "predict upload: %s", err.c_str());
    if (wide.empty()) return sync_stream(ctx);
    std::vector<int32_t> bigidx((size_t)p, -1);
    int nbig = 0;
    for (int64_t e : wide)
        if (bigidx[(size_t)(e % p)] < 0) bigidx[(size_t)(e % p)] = nbig++;
    TRY(sync_stream(ctx));
    TRY(predict_top_alloc(ctx, bigidx, nbig));
    return set_top_bits(ctx, wide, p, bigidx, n, ctx->d_ptopbits);
}

int gbm_predict_upload_raw(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype, const double *edges,
                           int32_t stride, const int32_t *counts, const int32_t *nan_bin) {
    if (!ctx || !X || !edges || !counts || !nan_bin || n <= 0 || p <= 0) return GBM_ERR_ARG;
    TRY(predict_alloc(ctx, n, p));
    std::vector<int32_t> bigidx((size_t)p, -1);
    int nbig = 0;
    for (int j = 0; j < p; j++)
        if (counts[j] > kBins) bigidx[(size_t)j] = nbig++;
    TRY(predict_top_alloc(ctx, bigidx, nbig));
    std::string err;
    if (gbmbin::bin_rows(ctx->bw, ctx->stager, ctx->st, X, n, p, dtype, edges, stride, counts, nan_bin, 0,
                         ctx->d_px, nbig ? ctx->d_pbigidx : nullptr, nbig ? ctx->d_ptopbits : nullptr, err))
        return bin_fail(ctx, err);
    return GBM_OK;
}

int gbm_predict_raw(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype, const double *edges,
                    int32_t stride, const int32_t *counts, const int32_t *nan_bin, const gbm_packed *model,
                    double lr, double base, double *F_out, double *proba_out) {
    TRY(gbm_predict_set_model(ctx, model, p));
    TRY(gbm_predict_upload_raw(ctx, X, n, p, dtype, edges, stride, counts, nan_bin));
    TRY(gbm_predict_run(ctx, lr, base));
    return gbm_predict_fetch(ctx, F_out, proba_out);
}

int gbm_predict_run(gbm_ctx *ctx, double lr, double base) {
    if (!ctx) return GBM_ERR_ARG;
    if (!ctx->d_px || !ctx->d_poff) return fail(ctx, GBM_ERR_STATE, "upload a model and rows first");
    // the packed walk reads a feature's byte unclamped: the rows must have the model's features
    if (ctx->pp != ctx->p_nfeat)
        return fail(ctx, GBM_ERR_ARG, "the rows have %d features, the model %d", ctx->pp, ctx->p_nfeat);
    CK(cudaSetDevice(ctx->dev));
    CK(launch_predict(ctx->d_px, ctx->pn, ctx->pp, ctx->d_pnodes, ctx->p_packed, ctx->d_pvals, ctx->d_poff,
                      ctx->d_pdep, ctx->p_ntree, ctx->d_pchunk,
                      reinterpret_cast<const int32_t *>(ctx->d_pchunk + ctx->p_ntree + 1), lr, base, ctx->d_pF,
                      ctx->d_pP, ctx->p_top ? ctx->d_pbigidx : nullptr, ctx->p_top ? ctx->d_ptopbits : nullptr,
                      ctx->st, ctx->p_packed_nr));
    ctx->launches++;
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
    out->host_sample_ms = ctx->host_sample_ms;
    out->host_sync_ms = ctx->host_sync_ms;
    out->host_replay_ms = ctx->host_replay_ms;
    out->flush_ms = ctx->flush_ms;
    out->hist_updates = ctx->hist_updates;
    out->host_comm_ms = ctx->host_comm_ms;
    out->comm_ms = ctx->comm_ms;
    out->comm_bytes = ctx->comm_bytes;
    out->peer_wait_ms = 0.0;
    out->sampler_ms = ctx->samp_ms;
    out->sampler_stall_ms = ctx->samp_stall_ms;
    if (ctx->p2p && ctx->d_sync && cudaSetDevice(ctx->dev) == cudaSuccess) {
        unsigned long long ns = 0;
        if (cudaMemcpy(&ns, ctx->d_sync + ctx->p2p_n + kSyncWaitNs, sizeof ns, cudaMemcpyDeviceToHost) == cudaSuccess)
            out->peer_wait_ms = (double)ns * 1e-6 - ctx->peer_wait_base_ms;
    }
    return GBM_OK;
}

int gbm_reset_stats(gbm_ctx *ctx) {
    if (!ctx) return GBM_ERR_ARG;
    ctx->launches = ctx->hist_launches = ctx->hist_rows = ctx->waves = 0;
    ctx->hist_ms = ctx->alg_bytes = ctx->hist_updates = 0.0;
    ctx->host_sample_ms = ctx->host_sync_ms = ctx->host_replay_ms = ctx->flush_ms = ctx->host_comm_ms = 0.0;
    ctx->comm_ms = ctx->comm_bytes = ctx->samp_ms = ctx->samp_stall_ms = 0.0;
    if (ctx->p2p && ctx->d_sync && cudaSetDevice(ctx->dev) == cudaSuccess) {   // the counter only grows
        unsigned long long ns = 0;
        if (cudaMemcpy(&ns, ctx->d_sync + ctx->p2p_n + kSyncWaitNs, sizeof ns, cudaMemcpyDeviceToHost) == cudaSuccess)
            ctx->peer_wait_base_ms = (double)ns * 1e-6;
    }
    return GBM_OK;
}

int gbm_set_l2_flush(gbm_ctx *ctx, int64_t bytes) {
    if (!ctx || bytes < 0) return GBM_ERR_ARG;
    if (ctx->dev < 0) return GBM_ERR_STATE;
    CK(cudaSetDevice(ctx->dev));
    TRY(sync_stream(ctx));
    if (ctx->d_flush) { dfree(ctx, ctx->d_flush); ctx->d_flush = nullptr; }
    ctx->flush_bytes = 0;
    if (bytes > 0) {
        TRY(dalloc(ctx, &ctx->d_flush, (size_t)bytes));
        ctx->flush_bytes = (size_t)bytes;
    }
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

// ===========================================================================
// Predict that allocates nothing
// ===========================================================================
//
// Some callers cannot call cudaMalloc: a serving process whose device memory
// is one arena handed out by its own allocator, a framework that owns the
// whole GPU, or a latency-bound path where an allocation (which may
// synchronise the device) is not allowed.  gbm_predict_noalloc takes every
// input and output as a device pointer the caller already owns and keeps its
// only scratch -- the ensemble rewritten as 8-byte nodes, which the traversal
// reads far better than the reference's 18-byte packed arrays -- in the
// fixed device array below.  Every GPU that loads this library holds that
// array (4 MiB) until the process exits.

namespace {

constexpr int kNoAllocMaxNodes = 1 << 19;   // 524,288 nodes: 1000 full depth-8 trees fit
constexpr int kNoAllocMaxTrees = 1 << 16;   // 65,536 trees

struct NoAllocScratch {
    PNode nodes[kNoAllocMaxNodes];
    int4 chunks[kNoAllocMaxTrees + 1];      // the walk's chunks of whole trees
    int32_t nchunk;
    int bad;          // set by the conversion kernel when the model is malformed
};

static __device__ __align__(256) NoAllocScratch g_noalloc;

// Host-side addresses of g_noalloc, one per device.  In host code the name
// g_noalloc is only a stand-in for the symbol, so the device address is
// looked up once per device (with that device current) and cached.
std::mutex g_noalloc_mu;
NoAllocScratch *g_noalloc_ptr[64] = {};

// Packed ensemble (device arrays) -> 8-byte nodes in the scratch array, with
// the checks that make the traversal safe: features < p, thresholds in
// [0, 255], children inside their tree and after their parent (so every
// path ends), offsets non-decreasing and within the node count.
__global__ void k_noalloc_pack(const int16_t *__restrict__ feat, const int64_t *__restrict__ thr,
                               const int32_t *__restrict__ left, const int32_t *__restrict__ right,
                               const int32_t *__restrict__ off, int32_t n_trees, int32_t n_nodes, int32_t p,
                               NoAllocScratch *__restrict__ sc) {
    int t = blockIdx.x;
    if (t >= n_trees) return;
    int o = off[t], o1 = off[t + 1];
    if (o < 0 || o1 < o || o1 > n_nodes || o1 - o > 32767) {
        if (threadIdx.x == 0) sc->bad = 1;
        return;
    }
    if (o1 == o) {   // an empty tree would be read at its node 0
        if (threadIdx.x == 0) sc->bad = 1;
        return;
    }
    const int sz = o1 - o;
    for (int k = threadIdx.x; k < sz; k += blockDim.x) {
        int f = feat[o + k];
        PNode nd;
        nd.feat = (int16_t)f;
        nd.nanr = 0;
        nd.thr = 0;
        nd.left = nd.right = 0;
        if (f >= 0) {
            long long th = thr[o + k];
            int l = left[o + k], r = right[o + k];
            bool ok = f < p && th >= 0 && th <= 255 && l > k && l < sz && r > k && r < sz;
            if (!ok) {
                sc->bad = 1;
                nd.feat = -1;
            } else {
                nd.thr = (uint8_t)th;
                nd.left = (int16_t)l;
                nd.right = (int16_t)r;
            }
        }
        sc->nodes[o + k] = nd;
    }
}

int noalloc_fail(char *errbuf, int32_t errlen, int code, const char *msg) {
    if (errbuf && errlen > 0) {
        std::strncpy(errbuf, msg, (size_t)errlen - 1);
        errbuf[errlen - 1] = '\0';
    }
    return code;
}

}  // namespace

extern "C" {

// See include/gbm_b200.h.
int gbm_predict_noalloc(const uint8_t *xbin_dev, int64_t n, int32_t p, const int16_t *features_dev,
                        const int64_t *thresholds_dev, const double *values_dev, const int32_t *left_dev,
                        const int32_t *right_dev, const int32_t *offsets_dev, int32_t n_trees, int32_t n_nodes,
                        double learning_rate, double base_score, double *F_dev, double *proba_dev, void *stream,
                        char *errbuf, int32_t errlen) {
    if (!xbin_dev || n <= 0 || p <= 0 || n_trees <= 0 || !features_dev || !thresholds_dev || !values_dev ||
        !left_dev || !right_dev || !offsets_dev || (!F_dev && !proba_dev))
        return noalloc_fail(errbuf, errlen, GBM_ERR_ARG, "gbm_predict_noalloc: null pointer or empty size");
    if (n_nodes <= 0 || n_nodes > kNoAllocMaxNodes || n_trees > kNoAllocMaxTrees) {
        char m[200];
        snprintf(m, sizeof m, "gbm_predict_noalloc: %d trees of %d nodes; the fixed scratch holds at most %d trees "
                 "and %d nodes", n_trees, n_nodes, kNoAllocMaxTrees, kNoAllocMaxNodes);
        return noalloc_fail(errbuf, errlen, GBM_ERR_ARG, m);
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return noalloc_fail(errbuf, errlen, GBM_ERR_CUDA, "gbm_predict_noalloc: no current CUDA device");
    NoAllocScratch *sc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void *ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc);
            if (e != cudaSuccess || !ptr)
                return noalloc_fail(errbuf, errlen, GBM_ERR_CUDA,
                                    "gbm_predict_noalloc: cudaGetSymbolAddress of the scratch array failed");
            g_noalloc_ptr[dev] = static_cast<NoAllocScratch *>(ptr);
        }
        sc = g_noalloc_ptr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the array keeps the previous call's contents: clear the error flag
    cudaError_t e = cudaMemsetAsync(&sc->bad, 0, sizeof(int), st);
    if (e == cudaSuccess) {
        k_noalloc_pack<<<n_trees, 256, 0, st>>>(features_dev, thresholds_dev, left_dev, right_dev, offsets_dev,
                                                 n_trees, n_nodes, p, sc);
        e = cudaGetLastError();
    }
    int bad = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&bad, &sc->bad, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return noalloc_fail(errbuf, errlen, GBM_ERR_CUDA, cudaGetErrorString(e));
    if (bad)
        return noalloc_fail(errbuf, errlen, GBM_ERR_ARG,
                            "gbm_predict_noalloc: malformed ensemble (offsets, feature, threshold or child out "
                            "of range, or a child not after its parent)");
    k_pred_chunks<<<1, 32, 0, st>>>(offsets_dev, n_trees, sc->chunks, &sc->nchunk);
    e = cudaGetLastError();
    // the walk is bounded by each tree's own size (from offsets_dev, checked
    // above), so a call that overlaps this one and rewrites the shared nodes
    // can make this one's output wrong but cannot send it outside the arrays
    if (e == cudaSuccess)
        e = launch_predict(xbin_dev, n, p, sc->nodes, false, values_dev, offsets_dev, nullptr, n_trees, sc->chunks,
                           &sc->nchunk, learning_rate, base_score, F_dev, proba_dev, nullptr, nullptr, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return noalloc_fail(errbuf, errlen, GBM_ERR_CUDA, cudaGetErrorString(e));
    return GBM_OK;
}

}  // extern "C"
