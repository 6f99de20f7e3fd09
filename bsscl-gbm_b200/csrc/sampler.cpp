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
// cache; a background thread runs rounds ahead, since the stream does not
// depend on the model.
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

struct MT19937 {
    uint32_t mt[624];
    int idx = 625;
    void seed(uint32_t s) {
        mt[0] = s;
        for (int i = 1; i < 624; i++) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
        idx = 624;
    }
    void twist() {
        for (int i = 0; i < 624; i++) {
            uint32_t y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
            uint32_t v = mt[(i + 397) % 624] ^ (y >> 1);
            if (y & 1u) v ^= 0x9908b0dfu;
            mt[i] = v;
        }
        idx = 0;
    }
    inline uint32_t next32() {
        if (idx >= 624) twist();
        uint32_t y = mt[idx++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        return y;
    }
    inline uint64_t next64() {
        uint64_t hi = next32();
        return (hi << 32) | next32();
    }
    // Uniform integer in [0, max] by masked rejection (NumPy legacy form).
    inline uint64_t interval(uint64_t max) {
        if (max == 0) return 0;
        uint64_t mask = max;
        mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4;
        mask |= mask >> 8; mask |= mask >> 16; mask |= mask >> 32;
        uint64_t v;
        if (max <= 0xffffffffull) {
            while ((v = (next32() & mask)) > max) {}
        } else {
            while ((v = (next64() & mask)) > max) {}
        }
        return v;
    }
};

template <typename T>
void shuffle(MT19937 &r, T *a, int64_t n) {
    for (int64_t i = n - 1; i >= 1; i--) {
        int64_t j = (int64_t)r.interval((uint64_t)i);
        T t = a[i]; a[i] = a[j]; a[j] = t;
    }
}

struct Draw {
    std::vector<int32_t> sample;   // n_sub row ids in the reference's order
    std::vector<int32_t> feat;     // n_feat sorted feature ids
};

}  // namespace

struct gbm_sampler {
    MT19937 rng;
    int64_t n = 0, n_sub = 0;
    int32_t p = 0, n_feat = 0;
    int sub_on = 0, col_on = 0;
    std::vector<int32_t> perm;
    std::vector<int32_t> fperm;
    // look-ahead
    int ahead = 0;
    std::thread worker;
    std::mutex mu;
    std::condition_variable cv;
    std::deque<Draw> q;
    bool stop = false;

    Draw make() {
        Draw d;
        if (sub_on) shuffle(rng, perm.data(), n);
        d.sample.assign(perm.begin(), perm.begin() + n_sub);
        if (col_on) shuffle(rng, fperm.data(), p);
        d.feat.assign(fperm.begin(), fperm.begin() + n_feat);
        std::sort(d.feat.begin(), d.feat.end());
        return d;
    }
    void run() {
        for (;;) {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return stop || (int)q.size() < ahead; });
            if (stop) return;
            lk.unlock();
            Draw d = make();
            lk.lock();
            q.push_back(std::move(d));
            cv.notify_all();
        }
    }
    Draw next() {
        if (ahead <= 0) return make();
        std::unique_lock<std::mutex> lk(mu);
        cv.wait(lk, [&] { return !q.empty(); });
        Draw d = std::move(q.front());
        q.pop_front();
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
    if (s->ahead > 0) s->worker = std::thread([s] { s->run(); });
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

void gbm_sampler_destroy(gbm_sampler *s) {
    if (!s) return;
    if (s->worker.joinable()) {
        {
            std::lock_guard<std::mutex> lk(s->mu);
            s->stop = true;
        }
        s->cv.notify_all();
        s->worker.join();
    }
    delete s;
}

}  // extern "C"
