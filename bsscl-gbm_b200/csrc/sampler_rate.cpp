// sampler_rate.cpp -- how many rounds per second the bit-exact sampler can
// feed an engine (swap targets of 1M rows plus 70 of 100 features per
// round, one draw thread running ahead), and the single-thread draw time.
// Build and run: make -C bsscl-gbm_b200/csrc sampler_rate && bsscl-gbm_b200/csrc/sampler_rate
#include <chrono>
#include <cstdio>
#include <vector>

#include "sampler_internal.h"

int main() {
    using clk = std::chrono::steady_clock;
    const int64_t n = 1000000;
    for (int ahead : {0, 3}) {
        gbm_sampler *s = nullptr;
        if (gbm_sampler_create(0, n, 100, 750000, 70, 1, 1, ahead, &s) != GBM_OK) return 1;
        std::vector<int32_t> t((size_t)n + 16), f(70);
        for (int k = 0; k < 5; k++) gbm_sampler_take_targets(s, t.data(), f.data());
        const int K = 100;
        auto t0 = clk::now();
        for (int k = 0; k < K; k++) gbm_sampler_take_targets(s, t.data(), f.data());
        double ms = std::chrono::duration<double, std::milli>(clk::now() - t0).count() / K;
        printf("look_ahead=%d: %.3f ms per round (%.0f rounds/s)\n", ahead, ms, 1000.0 / ms);
        gbm_sampler_destroy(s);
    }
    return 0;
}
