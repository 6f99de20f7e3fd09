// h2d.cpp -- see h2d.h.
#include "h2d.h"

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace gbmh2d {

namespace {

constexpr int kBufs = 3;                  // pinned buffers in the ring
constexpr size_t kChunk = 32u << 20;      // bytes per pinned buffer

// Narrowing also records, in `wide`, the element index (first_elem + i)
// of every value above 255 (rare: the top bin of 257-bin features).
void pack_range(const uint8_t *src, uint8_t *dst, size_t nsrc, Pack pk, int64_t first_elem,
                std::vector<int64_t> *wide) {
    if (pk == Pack::Copy) {
        std::memcpy(dst, src, nsrc);
        return;
    }
    const uint16_t *s = reinterpret_cast<const uint16_t *>(src);
    const size_t m = nsrc / 2;
    for (size_t i = 0; i < m; i++) {
        const uint16_t v = s[i];
        if (v > 255) {
            if (wide) wide->push_back(first_elem + (int64_t)i);
            dst[i] = 255;
        } else {
            dst[i] = (uint8_t)v;
        }
    }
}

}  // namespace

struct Stager {
    uint8_t *pin[kBufs] = {};
    cudaEvent_t ev[kBufs] = {};
    bool used[kBufs] = {};
    bool ready = false;

    // worker pool: part 0 of a job runs on the calling thread, part k on worker k-1
    int parts = 1;
    std::vector<std::thread> workers;
    std::mutex mu;
    std::condition_variable go_cv, done_cv;
    unsigned long long gen = 0;
    int pending = 0;
    bool stop = false;
    const uint8_t *jsrc = nullptr;
    uint8_t *jdst = nullptr;
    size_t jn = 0;
    Pack jpk = Pack::Copy;
    int64_t jelem = 0;                        // element index of jsrc in the whole matrix
    std::vector<int64_t> *jwide = nullptr;    // narrowed values above 255 (element indices)
    mutable std::mutex wmu;

    void part(int k) const {
        // parts start on 64-byte source boundaries (whole uint16 values)
        const size_t per = ((jn / (size_t)parts) + 63) & ~(size_t)63;
        const size_t a = std::min(jn, per * (size_t)k), b = std::min(jn, per * (size_t)(k + 1));
        const size_t div = jpk == Pack::U16toU8 ? 2 : 1;
        if (b > a) {
            std::vector<int64_t> local;
            pack_range(jsrc + a, jdst + a / div, b - a, jpk, jelem + (int64_t)(a / 2), jwide ? &local : nullptr);
            if (!local.empty()) {
                std::lock_guard<std::mutex> lk(wmu);
                jwide->insert(jwide->end(), local.begin(), local.end());
            }
        }
    }

    void worker(int k) {
        unsigned long long seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu);
                go_cv.wait(lk, [&] { return stop || gen != seen; });
                if (stop) return;
                seen = gen;
            }
            part(k);
            {
                std::lock_guard<std::mutex> lk(mu);
                if (--pending == 0) done_cv.notify_one();
            }
        }
    }

    void run(const uint8_t *src, uint8_t *dst, size_t n, Pack pk, int64_t elem0, std::vector<int64_t> *wide) {
        jsrc = src;
        jdst = dst;
        jn = n;
        jpk = pk;
        jelem = elem0;
        jwide = wide;
        if (parts == 1 || n < (1u << 20)) {
            const int saved = parts;
            parts = 1;
            part(0);
            parts = saved;
            return;
        }
        {
            std::lock_guard<std::mutex> lk(mu);
            pending = parts - 1;
            gen++;
        }
        go_cv.notify_all();
        part(0);
        std::unique_lock<std::mutex> lk(mu);
        done_cv.wait(lk, [&] { return pending == 0; });
    }
};

Stager *stager_create() {
    Stager *s = new Stager();
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    s->parts = (int)std::min(8u, std::max(1u, hw / 2));
    for (int k = 1; k < s->parts; k++) s->workers.emplace_back([s, k] { s->worker(k); });
    return s;
}

void stager_destroy(Stager *s) {
    if (!s) return;
    {
        std::lock_guard<std::mutex> lk(s->mu);
        s->stop = true;
    }
    s->go_cv.notify_all();
    for (auto &t : s->workers) t.join();
    for (int k = 0; k < kBufs; k++) {
        if (s->ev[k]) {
            cudaEventSynchronize(s->ev[k]);
            cudaEventDestroy(s->ev[k]);
        }
        if (s->pin[k]) cudaFreeHost(s->pin[k]);
    }
    delete s;
}

size_t chunk_bytes() { return kChunk; }

int stream_rows(Stager *s, cudaStream_t st, const void *src, int64_t rows, size_t row_bytes, Pack pack,
                int64_t max_chunk_rows, const std::function<void *(int64_t, int64_t)> &dst,
                const std::function<int(int64_t, int64_t, const void *)> &after, std::string &err,
                std::vector<int64_t> *wide) {
    if (rows <= 0) return 0;
    const size_t out_row = pack == Pack::U16toU8 ? row_bytes / 2 : row_bytes;
    if (out_row == 0 || out_row > kChunk) {
        err = "row too large for the upload buffers";
        return -1;
    }
    if (!s->ready) {
        for (int k = 0; k < kBufs; k++) {
            cudaError_t e = cudaHostAlloc(reinterpret_cast<void **>(&s->pin[k]), kChunk, cudaHostAllocPortable);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->ev[k], cudaEventDisableTiming);
            if (e != cudaSuccess) {
                err = std::string("pinned upload buffers: ") + cudaGetErrorString(e);
                return -1;
            }
        }
        s->ready = true;
    }
    int64_t cr = (int64_t)(kChunk / out_row);
    if (max_chunk_rows > 0) cr = std::min(cr, max_chunk_rows);
    const uint8_t *base = static_cast<const uint8_t *>(src);
    int c = 0;
    for (int64_t r0 = 0; r0 < rows; r0 += cr, c++) {
        const int64_t nr = std::min(cr, rows - r0);
        const int k = c % kBufs;
        if (s->used[k]) {
            cudaError_t e = cudaEventSynchronize(s->ev[k]);
            if (e != cudaSuccess) {
                err = std::string("upload: ") + cudaGetErrorString(e);
                return -1;
            }
        }
        s->run(base + (size_t)r0 * row_bytes, s->pin[k], (size_t)nr * row_bytes, pack,
               (int64_t)((size_t)r0 * row_bytes / 2), pack == Pack::U16toU8 ? wide : nullptr);
        void *d = dst(r0, nr);
        cudaError_t e = cudaMemcpyAsync(d, s->pin[k], (size_t)nr * out_row, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaEventRecord(s->ev[k], st);
        if (e != cudaSuccess) {
            err = std::string("upload: ") + cudaGetErrorString(e);
            return -1;
        }
        s->used[k] = true;
        if (after && after(r0, nr, d) != 0) return -1;
    }
    return 0;
}

}  // namespace gbmh2d
