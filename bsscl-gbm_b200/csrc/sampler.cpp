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
// The stream does not depend on the model, so a host thread draws rounds
// ahead.  For an engine only the swap targets leave this file: the engine
// turns them into the round's permutation on the GPU (the sequential
// MT19937 draw is all that stays on the host).  gbm_sampler_next applies
// the swaps to a host copy of the permutation (int32, n < 2^31).
#include <immintrin.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "../../include/gbm_b200.h"
#include "sampler_internal.h"

namespace gbmsamp {

constexpr int kN = 624, kM = 397;

// AVX-512 (F, BW, VL, DQ) versions of the twist and of the target draw are
// used when the CPU has them (the B200 hosts' Xeons do); GBM_SAMPLER_ISA=avx2
// forces the AVX2 versions.  Both give the same words and targets.
#define GBM_AVX512 __attribute__((target("avx512f,avx512bw,avx512vl,avx512dq")))

bool use_avx512() {
    static const bool on = [] {
        const char *e = std::getenv("GBM_SAMPLER_ISA");
        if (e && std::strcmp(e, "avx2") == 0) return false;
        __builtin_cpu_init();
        return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
               __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512dq");
    }();
    return on;
}

// The MT19937 twist and tempering, 16 words at a time.  The first 227 words
// read only old state, the next 396 read words this twist already wrote
// (i - 227 < i), and word 623 reads the new word 0.
GBM_AVX512 static inline __m512i mix16(__m512i a, __m512i b, __m512i c) {
    const __m512i y = _mm512_or_si512(_mm512_and_si512(a, _mm512_set1_epi32((int)0x80000000u)),
                                      _mm512_and_si512(b, _mm512_set1_epi32(0x7fffffff)));
    const __m512i r = _mm512_xor_si512(c, _mm512_srli_epi32(y, 1));
    return _mm512_mask_xor_epi32(r, _mm512_test_epi32_mask(y, _mm512_set1_epi32(1)), r,
                                 _mm512_set1_epi32((int)0x9908b0dfu));
}

static inline uint32_t mix1(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t y = (a & 0x80000000u) | (b & 0x7fffffffu);
    return c ^ (y >> 1) ^ ((0u - (y & 1u)) & 0x9908b0dfu);
}

GBM_AVX512 void twist_avx512(uint32_t *mt, uint32_t *out) {
    int i = 0;
    for (; i + 16 <= kN - kM; i += 16)
        _mm512_storeu_si512(mt + i, mix16(_mm512_loadu_si512(mt + i), _mm512_loadu_si512(mt + i + 1),
                                          _mm512_loadu_si512(mt + i + kM)));
    for (; i < kN - kM; i++) mt[i] = mix1(mt[i], mt[i + 1], mt[i + kM]);
    for (; i + 16 <= kN - 1; i += 16)
        _mm512_storeu_si512(mt + i, mix16(_mm512_loadu_si512(mt + i), _mm512_loadu_si512(mt + i + 1),
                                          _mm512_loadu_si512(mt + i + kM - kN)));
    for (; i < kN - 1; i++) mt[i] = mix1(mt[i], mt[i + 1], mt[i + kM - kN]);
    mt[kN - 1] = mix1(mt[kN - 1], mt[0], mt[kM - 1]);
    const __m512i t1 = _mm512_set1_epi32((int)0x9d2c5680u), t2 = _mm512_set1_epi32((int)0xefc60000u);
    for (int k = 0; k < kN; k += 16) {
        __m512i y = _mm512_loadu_si512(mt + k);
        y = _mm512_xor_si512(y, _mm512_srli_epi32(y, 11));
        y = _mm512_xor_si512(y, _mm512_and_si512(_mm512_slli_epi32(y, 7), t1));
        y = _mm512_xor_si512(y, _mm512_and_si512(_mm512_slli_epi32(y, 15), t2));
        y = _mm512_xor_si512(y, _mm512_srli_epi32(y, 18));
        _mm512_storeu_si512(out + k, y);
    }
}

// One twist of MT19937 state `mt`, tempered into dst[0 .. kN).
void twist_into(uint32_t *mt, uint32_t *dst) {
    if (use_avx512()) {
        twist_avx512(mt, dst);
        return;
    }
    int i = 0;
    for (; i < kN - kM; i++) mt[i] = mix1(mt[i], mt[i + 1], mt[i + kM]);
    for (; i < kN - 1; i++) mt[i] = mix1(mt[i], mt[i + 1], mt[i + kM - kN]);
    mt[kN - 1] = mix1(mt[kN - 1], mt[0], mt[kM - 1]);
    for (int k = 0; k < kN; k++) {
        uint32_t y = mt[k];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        dst[k] = y;
    }
}

// The words of a stream ahead of its draws, made by a second thread.  The
// MT19937 word stream does not depend on the draws that consume it, so a
// generator thread twists and tempers it into a ring of chunks while the
// draw thread decides targets from the chunks in order: the same words in
// the same order, with the twist off the draw's critical path.
struct WordPipe {
    static constexpr int kTwists = 16;                 // twists per chunk
    static constexpr int kChunkWords = kTwists * kN;   // 9984 words (39 KB)
    static constexpr int kChunks = 48;                 // a 1.9 MB ring
    uint32_t mt[kN];                                   // the generator's state
    std::vector<uint32_t> ring;
    std::atomic<int64_t> made{0}, freed{0};           // chunks written / released by the reader
    std::atomic<bool> stop{false};
    int64_t cur = -1;                                  // the reader's chunk
    std::thread th;

    explicit WordPipe(const uint32_t *state) : ring((size_t)kChunks * kChunkWords) {
        std::memcpy(mt, state, sizeof mt);
        th = std::thread([this] { run(); });
    }
    ~WordPipe() {
        stop.store(true);
        if (th.joinable()) th.join();
    }
    void run() {
        int idle = 0;   // polls of a full ring in a row: spin while the reader is active, then sleep
        while (!stop.load(std::memory_order_relaxed)) {
            const int64_t h = made.load(std::memory_order_relaxed);
            if (h - freed.load(std::memory_order_acquire) >= kChunks) {   // full: the reader is behind
                if (++idle < (1 << 16)) _mm_pause();
                else std::this_thread::sleep_for(std::chrono::microseconds(200));
                continue;
            }
            idle = 0;
            uint32_t *dst = ring.data() + (size_t)(h % kChunks) * kChunkWords;
            for (int k = 0; k < kTwists; k++) twist_into(mt, dst + k * kN);
            made.store(h + 1, std::memory_order_release);
        }
    }
    // The reader: release the current chunk and wait for the next.
    const uint32_t *next() {
        if (cur >= 0) freed.store(cur + 1, std::memory_order_release);
        cur++;
        int spins = 0;
        while (made.load(std::memory_order_acquire) <= cur) {
            if (++spins < 512) _mm_pause();
            else std::this_thread::yield();
        }
        return ring.data() + (size_t)(cur % kChunks) * kChunkWords;
    }
};

// The reader's view of the stream: a window out[0 .. len) of tempered
// words, refilled by one twist, or by the next chunk of a WordPipe.
struct MT19937 {
    uint32_t mt[kN];
    uint32_t buf[kN];
    const uint32_t *out = buf;
    int idx = kN, len = kN;
    WordPipe *pipe = nullptr;
    void seed(uint32_t s) {
        mt[0] = s;
        for (int i = 1; i < kN; i++) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
        idx = len = kN;
        out = buf;
    }
    void refill() {
        if (pipe) {
            out = pipe->next();
            len = WordPipe::kChunkWords;
        } else {
            twist_into(mt, buf);
            out = buf;
            len = kN;
        }
        idx = 0;
    }
    inline uint32_t next32() {
        if (idx >= len) refill();
        return out[idx++];
    }
};

// The compress permutations of AVX2 left-packing: entry m lists the lanes
// whose bit is set in m, in order.
struct CompressLut {
    alignas(32) int32_t idx[256][8];
    CompressLut() {
        for (int m = 0; m < 256; m++) {
            int k = 0;
            for (int l = 0; l < 8; l++)
                if (m & (1 << l)) idx[m][k++] = l;
            for (; k < 8; k++) idx[m][k] = 0;
        }
    }
};
const CompressLut kLut;

inline uint32_t smear(uint64_t i) {
    uint32_t m = (uint32_t)i;
    m |= m >> 1; m |= m >> 2; m |= m >> 4; m |= m >> 8; m |= m >> 16;
    return m;
}

// Swap targets of NumPy's legacy shuffle for i = n-1 .. 1, stored forward:
// t[k] is the target of i = n-1-k (k = 0 .. n-2).
// Each target is a uniform integer in [0, i] drawn by masked rejection (the
// smallest all-ones mask covering i, one 32-bit word per attempt, rejected
// if > i).  The words are consumed in the scalar rule's order, but a block
// of B words is decided at once when no word of it lies in (i-B+1, i]: each
// word is then > i (rejected whatever the others do) or <= i-B+1 (accepted),
// and i-B+1 still has the block's mask.  Accepted words are left-packed into
// t (AVX2, 8 lanes).  Blocks of 64, then 8, then single words.
inline void pack8(__m256i v, int nacc, int32_t *t, int64_t &pos) {
    const int acc = ~nacc & 0xff;
    const __m256i pm = _mm256_load_si256((const __m256i *)kLut.idx[acc]);
    _mm256_storeu_si256((__m256i *)(t + pos), _mm256_permutevar8x32_epi32(v, pm));
    pos += __builtin_popcount((unsigned)acc);
}

GBM_AVX512 void draw_targets_avx512(MT19937 &r, int64_t n, int32_t *t) {
    const int64_t top = n - 1;
    int64_t pos = 0;                    // i = top - pos
    while (top - pos >= 1) {
        if (r.idx >= r.len) r.refill();
        int64_t i = top - pos;
        const uint32_t mask = smear((uint64_t)i);
        const int64_t stop = ((int64_t)mask + 1) >> 1;   // lowest i with this mask
        const uint32_t *w = r.out;
        const int L = r.len;
        int k = r.idx;
        const __m512i vm = _mm512_set1_epi32((int)mask);
        // 64-word blocks: four independent compares, one store chain
        while (k + 64 <= L && i - 63 >= stop) {
            const __m512i hi = _mm512_set1_epi32((int)i), lo = _mm512_set1_epi32((int)(i - 63));
            __m512i v[4];
            __mmask16 nacc[4];
            unsigned amb = 0;
            for (int b = 0; b < 4; b++) {
                v[b] = _mm512_and_si512(_mm512_loadu_si512(w + k + 16 * b), vm);
                const __mmask16 rej = _mm512_cmpgt_epi32_mask(v[b], hi);
                nacc[b] = _mm512_cmpgt_epi32_mask(v[b], lo);
                amb |= (unsigned)(nacc[b] & (__mmask16)~rej);
            }
            if (amb) break;
            for (int b = 0; b < 4; b++) {
                const __mmask16 acc = (__mmask16)~nacc[b];
                _mm512_storeu_si512(t + pos, _mm512_maskz_compress_epi32(acc, v[b]));
                pos += __builtin_popcount((unsigned)acc);
            }
            k += 64;
            i = top - pos;
        }
        // 16-word blocks (at most 4 of them before trying 64 again)
        for (int blk = 0; blk < 4 && k + 16 <= L && i - 15 >= stop; blk++) {
            const __m512i v = _mm512_and_si512(_mm512_loadu_si512(w + k), vm);
            const __mmask16 rej = _mm512_cmpgt_epi32_mask(v, _mm512_set1_epi32((int)i));
            const __mmask16 nacc = _mm512_cmpgt_epi32_mask(v, _mm512_set1_epi32((int)(i - 15)));
            if (nacc & (__mmask16)~rej) break;
            const __mmask16 acc = (__mmask16)~nacc;
            _mm512_storeu_si512(t + pos, _mm512_maskz_compress_epi32(acc, v));
            pos += __builtin_popcount((unsigned)acc);
            k += 16;
            i = top - pos;
        }
        // single words, up to 16
        const int end = std::min(L, k + 16);
        while (k < end && i >= stop) {
            const uint32_t v = w[k++] & mask;
            t[pos] = (int32_t)v;
            const int64_t a = (int64_t)(v <= (uint64_t)i);
            pos += a;
            i -= a;
        }
        r.idx = k;
    }
}

void draw_targets_avx2(MT19937 &r, int64_t n, int32_t *t) {
    const int64_t top = n - 1;
    int64_t pos = 0;                    // i = top - pos
    while (top - pos >= 1) {
        if (r.idx >= r.len) r.refill();
        int64_t i = top - pos;
        const uint32_t mask = smear((uint64_t)i);
        const int64_t stop = ((int64_t)mask + 1) >> 1;   // lowest i with this mask
        const uint32_t *w = r.out;
        const int L = r.len;
        int k = r.idx;
        const __m256i vm = _mm256_set1_epi32((int)mask);
        // 64-word blocks: eight independent compares, one store chain
        while (k + 64 <= L && i - 63 >= stop) {
            const __m256i hi = _mm256_set1_epi32((int)i), lo = _mm256_set1_epi32((int)(i - 63));
            __m256i v[8];
            int nacc[8], amb = 0;
            for (int b = 0; b < 8; b++) {
                v[b] = _mm256_and_si256(_mm256_loadu_si256((const __m256i *)(w + k + 8 * b)), vm);
                const int rej = _mm256_movemask_ps(_mm256_castsi256_ps(_mm256_cmpgt_epi32(v[b], hi)));
                nacc[b] = _mm256_movemask_ps(_mm256_castsi256_ps(_mm256_cmpgt_epi32(v[b], lo)));
                amb |= nacc[b] & ~rej;
            }
            if (amb) break;
            for (int b = 0; b < 8; b++) pack8(v[b], nacc[b], t, pos);
            k += 64;
            i = top - pos;
        }
        // 8-word blocks (at most 8 of them before trying 64 again)
        for (int blk = 0; blk < 8 && k + 8 <= L && i - 7 >= stop; blk++) {
            const __m256i v = _mm256_and_si256(_mm256_loadu_si256((const __m256i *)(w + k)), vm);
            const int rej = _mm256_movemask_ps(_mm256_castsi256_ps(_mm256_cmpgt_epi32(v, _mm256_set1_epi32((int)i))));
            const int nacc =
                _mm256_movemask_ps(_mm256_castsi256_ps(_mm256_cmpgt_epi32(v, _mm256_set1_epi32((int)(i - 7)))));
            if (nacc & ~rej) break;
            pack8(v, nacc, t, pos);
            k += 8;
            i = top - pos;
        }
        // single words, up to 8
        const int end = std::min(L, k + 8);
        while (k < end && i >= stop) {
            const uint32_t v = w[k++] & mask;
            t[pos] = (int32_t)v;
            const int64_t a = (int64_t)(v <= (uint64_t)i);
            pos += a;
            i -= a;
        }
        r.idx = k;
    }
}

// t holds n + 16 entries (the last block store may run past n - 1).
void draw_targets(MT19937 &r, int64_t n, int32_t *t) {
    if (use_avx512()) draw_targets_avx512(r, n, t);
    else draw_targets_avx2(r, n, t);
}

// Fisher-Yates from the last element down to index 1 (forward targets),
// targets prefetched.
template <typename T>
void apply_swaps(T *a, int64_t n, const int32_t *t) {
    constexpr int64_t kAhead = 24;
    for (int64_t k = 0; k + 1 < n; k++) {
        if (k + kAhead + 1 < n) __builtin_prefetch(&a[t[k + kAhead]], 1, 0);
        const int64_t i = n - 1 - k, j = t[k];
        T x = a[i]; a[i] = a[j]; a[j] = x;
    }
}

// One round drawn ahead: the row swap targets (the row shuffle itself is
// applied by the consumer: on the host for gbm_sampler_next, on the device
// for an engine) and the round's sorted feature ids.
struct Round {
    std::vector<int32_t> trow;          // n + 16 entries
    std::vector<int32_t> feat;          // n_feat
    bool ready = false;
};

enum { kModeUnset = 0, kModeHost, kModeTargets };

}  // namespace gbmsamp

using namespace gbmsamp;

struct gbm_sampler {
    MT19937 rng;
    std::unique_ptr<WordPipe> pipe;    // the words ahead (large draws drawn ahead only)
    int64_t n = 0, n_sub = 0;
    int32_t p = 0, n_feat = 0;
    int sub_on = 0, col_on = 0;
    // throughput mode (gbm_sampler_create_device): rows are drawn on the
    // device from a counter-based hash, in-bag iff hash < dev_thr
    int dev_rows = 0;
    uint64_t dev_seed = 0, dev_thr = 0;
    std::vector<int32_t> perm;         // host-side row permutation (kModeHost)
    std::vector<int32_t> fperm, tfeat;
    std::vector<int32_t> sample;
    int mode = kModeUnset;
    int64_t taken = 0;                 // rounds handed out
    Round sync_round;
    int ahead = 0;
    std::vector<Round> ring;
    int64_t r_draw = 0;
    std::thread t_draw;
    std::mutex mu;
    std::condition_variable cv;
    bool stop = false;

    // The round's row targets, and its feature shuffle (applied here: it is
    // cheap and must follow round order, as the draws do).
    void draw(Round &R) {
        if (sub_on) draw_targets(rng, n, R.trow.data());
        if (col_on) {
            draw_targets(rng, p, tfeat.data());
            apply_swaps(fperm.data(), p, tfeat.data());
        }
        std::memcpy(R.feat.data(), fperm.data(), sizeof(int32_t) * (size_t)n_feat);
        std::sort(R.feat.begin(), R.feat.end());
    }
    Round &slot(int64_t r) { return ring[(size_t)(r % (int64_t)ring.size())]; }
    void run_draw() {
        for (;;) {
            Round *R;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return stop || !slot(r_draw).ready; });
                if (stop) return;
                R = &slot(r_draw);
            }
            draw(*R);
            std::lock_guard<std::mutex> lk(mu);
            R->ready = true;
            r_draw++;
            cv.notify_all();
        }
    }
    // Hand the next round to `take` (called without the lock, before the
    // round's buffers are reused).
    template <typename F>
    void next(F &&take) {
        if (ahead <= 0) {
            draw(sync_round);
            take(sync_round);
            taken++;
            return;
        }
        Round *R;
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return slot(taken).ready; });
            R = &slot(taken);
        }
        take(*R);
        std::lock_guard<std::mutex> lk(mu);
        R->ready = false;
        taken++;
        cv.notify_all();
    }
    bool claim(int m) {
        if (mode == kModeUnset) mode = m;
        return mode == m;
    }
    // host mode: the cumulative shuffle of the rows, in place
    void host_sample(const Round &R) {
        if (sub_on) apply_swaps(perm.data(), n, R.trow.data());
        std::memcpy(sample.data(), perm.data(), sizeof(int32_t) * (size_t)n_sub);
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
    try {
        s->rng.seed(seed);
        s->n = n; s->p = p; s->n_sub = n_sub; s->n_feat = n_feat;
        s->sub_on = subsample_on; s->col_on = colsample_on;
        s->fperm.resize((size_t)p);
        for (int32_t i = 0; i < p; i++) s->fperm[(size_t)i] = i;
        s->tfeat.resize((size_t)p + 16);
        s->ahead = look_ahead < 0 ? 0 : look_ahead;
        auto size_round = [&](Round &R) {
            if (s->sub_on) R.trow.resize((size_t)n + 16);
            R.feat.resize((size_t)n_feat);
        };
        // a draw of a million rows spends about half its time in the twist:
        // drawn ahead, it gets a generator thread of its own
        if (s->ahead > 0 && n >= (1 << 17)) {
            s->pipe.reset(new WordPipe(s->rng.mt));
            s->rng.pipe = s->pipe.get();
        }
        if (s->ahead > 0) {
            s->ring.resize((size_t)s->ahead + 1);
            for (auto &R : s->ring) size_round(R);
            s->t_draw = std::thread([s] { s->run_draw(); });
        } else {
            size_round(s->sync_round);
        }
    } catch (...) {
        gbm_sampler_destroy(s);
        return GBM_ERR_ALLOC;
    }
    *out = s;
    return GBM_OK;
}

int gbm_sampler_create_device(uint32_t seed, int64_t n, int32_t p, double subsample, int32_t n_feat,
                              int32_t colsample_on, int32_t look_ahead, gbm_sampler **out) {
    if (!out || !(subsample > 0.0 && subsample <= 1.0)) return GBM_ERR_ARG;
    const int64_t n_sub = std::max<int64_t>(1, (int64_t)((double)n * subsample));
    int rc = gbm_sampler_create(seed, n, p, n_sub > n ? n : n_sub, n_feat, 0, colsample_on, look_ahead, out);
    if (rc != GBM_OK) return rc;
    gbm_sampler *s = *out;
    s->dev_rows = 1;
    s->dev_seed = 0x9e3779b97f4a7c15ull * ((uint64_t)seed + 1u);
    // in-bag iff hash < subsample * 2^64 (every row when subsample is 1)
    s->dev_thr = subsample >= 1.0 ? ~0ull : (uint64_t)std::ldexp(subsample, 64);
    return GBM_OK;
}

// Host outputs: the row permutation is kept here (first call decides).
static int host_ready(gbm_sampler *s) {
    if (s->dev_rows) return GBM_ERR_STATE;   // its rows are drawn on the device only
    if (!s->claim(kModeHost)) return GBM_ERR_STATE;
    if (s->perm.empty()) {
        try {
            s->perm.resize((size_t)s->n);
            s->sample.resize((size_t)s->n_sub);
        } catch (...) {
            return GBM_ERR_ALLOC;
        }
        for (int64_t i = 0; i < s->n; i++) s->perm[(size_t)i] = (int32_t)i;
    }
    return GBM_OK;
}

int gbm_sampler_next(gbm_sampler *s, int64_t *sample_idx, uint8_t *inbag_mask, int32_t *feat_idx) {
    if (!s) return GBM_ERR_ARG;
    int rc = host_ready(s);
    if (rc != GBM_OK) return rc;
    s->next([&](const Round &d) {
        s->host_sample(d);
        if (sample_idx)
            for (int64_t k = 0; k < s->n_sub; k++) sample_idx[k] = s->sample[(size_t)k];
        if (inbag_mask) {
            std::memset(inbag_mask, 0, (size_t)s->n);
            for (int64_t k = 0; k < s->n_sub; k++) inbag_mask[s->sample[(size_t)k]] = 1;
        }
        if (feat_idx)
            for (int32_t k = 0; k < s->n_feat; k++) feat_idx[k] = d.feat[(size_t)k];
    });
    return GBM_OK;
}

int gbm_sampler_next_rows(gbm_sampler *s, int32_t *sample_rows, int32_t *feat_idx) {
    if (!s || !sample_rows || !feat_idx) return GBM_ERR_ARG;
    int rc = host_ready(s);
    if (rc != GBM_OK) return rc;
    s->next([&](const Round &d) {
        s->host_sample(d);
        std::memcpy(sample_rows, s->sample.data(), sizeof(int32_t) * (size_t)s->n_sub);
        std::memcpy(feat_idx, d.feat.data(), sizeof(int32_t) * (size_t)s->n_feat);
    });
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
    delete s;
}

}  // extern "C"

// ---- engine side (sampler_internal.h) ----------------------------------------

int gbm_sampler_take_targets(gbm_sampler *s, int32_t *row_targets, int32_t *feat_idx) {
    if (!s || !feat_idx || (s->sub_on && !row_targets)) return GBM_ERR_ARG;
    if (!s->claim(kModeTargets)) return GBM_ERR_STATE;
    s->next([&](const Round &d) {
        if (s->sub_on) std::memcpy(row_targets, d.trow.data(), sizeof(int32_t) * (size_t)(s->n - 1));
        std::memcpy(feat_idx, d.feat.data(), sizeof(int32_t) * (size_t)s->n_feat);
    });
    return GBM_OK;
}

int64_t gbm_sampler_taken(const gbm_sampler *s) { return s ? s->taken : 0; }
int64_t gbm_sampler_rows(const gbm_sampler *s) { return s ? s->n : 0; }
int gbm_sampler_shuffles_rows(const gbm_sampler *s) { return s ? s->sub_on : 0; }
int gbm_sampler_device_rows(const gbm_sampler *s, uint64_t *seed, uint64_t *thr) {
    if (!s || !s->dev_rows) return 0;
    *seed = s->dev_seed;
    *thr = s->dev_thr;
    return 1;
}
