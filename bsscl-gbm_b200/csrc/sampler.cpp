// sampler.cpp -- the reference's per-round row/feature sampler, bit-exact.
//
// The reference draws each round's subsample with NumPy's legacy
// RandomState (src/bsscl_gbm/estimator_v1_0_1.py:3159) and, per round,
// shuffles a persistent int64 arange(n) in place and keeps the first n_sub
// entries, then shuffles a persistent int32 arange(p) and keeps the sorted
// first n_feat (E:2502-2517).  This file reimplements that stream natively:
//   * MT19937 (Matsumoto & Nishimura 1998) with the classic init_genrand
//     seeding that RandomState(int) uses;
//   * NumPy's legacy bounded integer draw for the shuffle: the smallest
//     all-ones mask covering `max`, 32-bit words, rejection of values > max;
//   * Fisher-Yates from the last element down to index 1.
// The permutation is kept as int32 (n < 2^31) so the 1M-row state fits in
// cache.  The stream does not depend on the model, so two host threads run
// rounds ahead: one draws the next round's swap targets (the whole MT19937
// cost), the other applies the previous round's swaps.
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "../../include/gbm_b200.h"

namespace {

constexpr int kN = 624, kM = 397;

struct MT19937 {
    uint32_t mt[kN];
    uint32_t out[kN];   // tempered words of the current state
    int idx = kN;
    void seed(uint32_t s) {
        mt[0] = s;
        for (int i = 1; i < kN; i++) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
        idx = kN;
    }
    static inline uint32_t mix(uint32_t a, uint32_t b, uint32_t c) {
        uint32_t y = (a & 0x80000000u) | (b & 0x7fffffffu);
        return c ^ (y >> 1) ^ ((0u - (y & 1u)) & 0x9908b0dfu);
    }
    void refill() {   // the standard twist (split so no index wraps), then tempering
        int i = 0;
        for (; i < kN - kM; i++) mt[i] = mix(mt[i], mt[i + 1], mt[i + kM]);
        for (; i < kN - 1; i++) mt[i] = mix(mt[i], mt[i + 1], mt[i + kM - kN]);
        mt[kN - 1] = mix(mt[kN - 1], mt[0], mt[kM - 1]);
        for (int k = 0; k < kN; k++) {
            uint32_t y = mt[k];
            y ^= y >> 11;
            y ^= (y << 7) & 0x9d2c5680u;
            y ^= (y << 15) & 0xefc60000u;
            y ^= y >> 18;
            out[k] = y;
        }
        idx = 0;
    }
    inline uint32_t next32() {
        if (idx >= kN) refill();
        return out[idx++];
    }
};

// Swap targets of NumPy's legacy shuffle for i = n-1 .. 1: each target is a
// uniform integer in [0, i] drawn by masked rejection (the smallest
// all-ones mask covering i, one 32-bit word per attempt, rejected if > i).
// The mask is constant for i in [2^(k-1), 2^k - 1], and the attempt loop is
// written without branches: every word is stored at tgt[i] and i only
// advances when the word was accepted -- the same words in the same order.
void draw_targets(MT19937 &r, int64_t n, int32_t *tgt) {
    int64_t i = n - 1;
    while (i >= 1) {
        if (r.idx >= kN) r.refill();
        uint32_t mask = (uint32_t)i;
        mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4;
        mask |= mask >> 8; mask |= mask >> 16;
        const int64_t stop = ((int64_t)mask + 1) >> 1;   // lowest i with this mask
        const uint32_t *w = r.out + r.idx;
        const int avail = kN - r.idx;
        int k = 0;
        while (k < avail && i >= stop) {
            uint32_t v = w[k++] & mask;
            tgt[i] = (int32_t)v;
            i -= (int64_t)(v <= (uint64_t)i);
        }
        r.idx += k;
    }
}

// Fisher-Yates from the last element down to index 1, targets prefetched.
template <typename T>
void apply_swaps(T *a, int64_t n, const int32_t *tgt) {
    constexpr int64_t kAhead = 24;
    for (int64_t i = n - 1; i >= 1; i--) {
        if (i > kAhead) __builtin_prefetch(&a[tgt[i - kAhead]], 1, 0);
        int64_t j = tgt[i];
        T t = a[i]; a[i] = a[j]; a[j] = t;
    }
}

struct Draw {
    std::vector<int32_t> sample;   // first n_sub of the permutation: sample_idx order
    std::vector<int32_t> feat;     // n_feat sorted feature ids
};

struct Targets {                   // one round's swap targets
    std::vector<int32_t> rows, feats;
};

}  // namespace

struct gbm_sampler {
    MT19937 rng;
    int64_t n = 0, n_sub = 0;
    int32_t p = 0, n_feat = 0;
    int sub_on = 0, col_on = 0;
    std::vector<int32_t> perm;
    std::vector<int32_t> fperm;
    Targets tg;                    // synchronous path scratch
    // look-ahead: stage 1 draws targets, stage 2 applies them
    int ahead = 0;
    std::thread t_draw, t_apply;
    std::mutex mu;
    std::condition_variable cv;
    std::deque<Targets> tq;
    std::deque<Draw> dq;
    bool stop = false;

    void make_targets(Targets &t) {
        if (sub_on) { t.rows.resize((size_t)n); draw_targets(rng, n, t.rows.data()); }
        if (col_on) { t.feats.resize((size_t)p); draw_targets(rng, p, t.feats.data()); }
    }
    Draw apply(const Targets &t) {
        Draw d;
        if (sub_on) apply_swaps(perm.data(), n, t.rows.data());
        d.sample.assign(perm.begin(), perm.begin() + n_sub);
        if (col_on) apply_swaps(fperm.data(), p, t.feats.data());
        d.feat.assign(fperm.begin(), fperm.begin() + n_feat);
        std::sort(d.feat.begin(), d.feat.end());
        return d;
    }
    void run_draw() {
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return stop || (int)tq.size() < ahead; });
                if (stop) return;
            }
            Targets t;
            make_targets(t);
            std::lock_guard<std::mutex> lk(mu);
            tq.push_back(std::move(t));
            cv.notify_all();
        }
    }
    void run_apply() {
        for (;;) {
            Targets t;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return stop || (!tq.empty() && (int)dq.size() < ahead); });
                if (stop) return;
                t = std::move(tq.front());
                tq.pop_front();
                cv.notify_all();
            }
            Draw d = apply(t);
            std::lock_guard<std::mutex> lk(mu);
            dq.push_back(std::move(d));
            cv.notify_all();
        }
    }
    Draw next() {
        if (ahead <= 0) {
            make_targets(tg);
            return apply(tg);
        }
        std::unique_lock<std::mutex> lk(mu);
        cv.wait(lk, [&] { return !dq.empty(); });
        Draw d = std::move(dq.front());
        dq.pop_front();
        cv.notify_all();
        return d;
    }
};

extern "C" {

int gbm_sampler_create(uint32_t seed, int64_t n, int32_t p, int64_t n_sub, int32_t n_feat,
                       int32_t subsample_on, int32_t colsample_on, int32_t look_ahead,
                       gbm_sampler **out) {
    if (!out || n <= 0 || n > 0x7fffffffLL || p <= 0 || n_sub <= 0 || n_sub > n ||
        n_feat <= 0 || n_feat > p)
        return GBM_ERR_ARG;
    gbm_sampler *s = new (std::nothrow) gbm_sampler();
    if (!s) return GBM_ERR_ALLOC;
    s->rng.seed(seed);
    s->n = n; s->p = p; s->n_sub = n_sub; s->n_feat = n_feat;
    s->sub_on = subsample_on; s->col_on = colsample_on;
    s->perm.resize((size_t)n);
    for (int64_t i = 0; i < n; i++) s->perm[(size_t)i] = (int32_t)i;
    s->fperm.resize((size_t)p);
    for (int32_t i = 0; i < p; i++) s->fperm[(size_t)i] = i;
    s->ahead = look_ahead < 0 ? 0 : look_ahead;
    if (s->ahead > 0) {
        s->t_draw = std::thread([s] { s->run_draw(); });
        s->t_apply = std::thread([s] { s->run_apply(); });
    }
    *out = s;
    return GBM_OK;
}

int gbm_sampler_next(gbm_sampler *s, int64_t *sample_idx, uint8_t *inbag_mask, int32_t *feat_idx) {
    if (!s) return GBM_ERR_ARG;
    Draw d = s->next();
    if (sample_idx)
        for (int64_t k = 0; k < s->n_sub; k++) sample_idx[k] = d.sample[(size_t)k];
    if (inbag_mask) {
        std::memset(inbag_mask, 0, (size_t)s->n);
        for (int64_t k = 0; k < s->n_sub; k++) inbag_mask[d.sample[(size_t)k]] = 1;
    }
    if (feat_idx)
        for (int32_t k = 0; k < s->n_feat; k++) feat_idx[k] = d.feat[(size_t)k];
    return GBM_OK;
}

int gbm_sampler_next_rows(gbm_sampler *s, int32_t *sample_rows, int32_t *feat_idx) {
    if (!s || !sample_rows || !feat_idx) return GBM_ERR_ARG;
    Draw d = s->next();
    std::memcpy(sample_rows, d.sample.data(), sizeof(int32_t) * (size_t)s->n_sub);
    std::memcpy(feat_idx, d.feat.data(), sizeof(int32_t) * (size_t)s->n_feat);
    return GBM_OK;
}

int64_t gbm_sampler_n_sub(const gbm_sampler *s) { return s ? s->n_sub : 0; }
int32_t gbm_sampler_n_feat(const gbm_sampler *s) { return s ? s->n_feat : 0; }

void gbm_sampler_destroy(gbm_sampler *s) {
    if (!s) return;
    {
        std::lock_guard<std::mutex> lk(s->mu);
        s->stop = true;
    }
    s->cv.notify_all();
    if (s->t_draw.joinable()) s->t_draw.join();
    if (s->t_apply.joinable()) s->t_apply.join();
    delete s;
}

}  // extern "C"
