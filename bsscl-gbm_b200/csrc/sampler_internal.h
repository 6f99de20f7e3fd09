// sampler_internal.h -- what the engine (gbm_b200.cu) reads from a sampler;
// not part of the C ABI (hidden in the shared library).
#pragma once
#include <cstdint>

#include "../../include/gbm_b200.h"

#define GBM_INTERNAL __attribute__((visibility("hidden")))

// The next round's row swap targets (t[k] is the target of i = n-1-k,
// k = 0 .. n-2; nothing when rows are not subsampled) and sorted feature
// ids.  A sampler used this way cannot also serve gbm_sampler_next.
GBM_INTERNAL int gbm_sampler_take_targets(gbm_sampler *s, int32_t *row_targets, int32_t *feat_idx);
GBM_INTERNAL int64_t gbm_sampler_taken(const gbm_sampler *s);
GBM_INTERNAL int64_t gbm_sampler_rows(const gbm_sampler *s);
GBM_INTERNAL int gbm_sampler_shuffles_rows(const gbm_sampler *s);
// 1 for a throughput-mode sampler (gbm_sampler_create_device): round r's
// in-bag rows are those with gbm_row_hash(seed, r, global row) < thr.
GBM_INTERNAL int gbm_sampler_device_rows(const gbm_sampler *s, uint64_t *seed, uint64_t *thr);
