// binning_internal.h -- bin edges and bin ids on the GPU (binning.cu), used
// by the C ABI in gbm_b200.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "h2d.h"

namespace gbmbin {

struct Work;   // device buffers of the binning pipeline, one per context

Work *work_create();
void work_destroy(Work *w);

// Uploads X (host, row-major [n][p]; dtype 0 = float32, 1 = float64) and
// keeps it on the device as column-major order keys for edges() and
// bin_blocks().
int load(Work *w, gbmh2d::Stager *sg, cudaStream_t st, const void *X, int64_t n, int p, int dtype,
         std::string &err);

// The loaded matrix's shape (false if none is loaded).
bool shape(const Work *w, int64_t &n, int &p);

// Frees the loaded matrix's keys and sort buffers.
void release(Work *w);

// Bin edges of the loaded matrix (HybridHistGBMNumbaV1_0_1._build_bin_edges,
// src/bsscl_gbm/estimator_v1_0_1.py:2073-2141, sample_weight=None), written
// to host memory as rows of `stride` float64 padded with each feature's last
// edge.  is_cat: NULL or [p] flags of categorical features.
int edges(Work *w, cudaStream_t st, int n_bins, const uint8_t *is_cat, double *edges_out, int stride,
          int32_t *counts_out, int32_t *nan_bin_out, int32_t *max_b_out, std::string &err);

// Bins rows [lo, hi) of the loaded matrix into the training layout: column
// blocks uint8 [ceil(p/16)][hi-lo][16], ids clamped to bin_count - 1; an id
// of 256 (a 257-bin feature) is stored as 255 and sets the row's bit in
// d_topbits [big feature d_bigidx[j]][ceil((hi - lo) / 32)] (zeroed by the
// caller).
int bin_blocks(Work *w, cudaStream_t st, int64_t lo, int64_t hi, const double *edges, int stride,
               const int32_t *counts, const int32_t *nan_bin, uint8_t *d_xb, const int32_t *d_bigidx,
               uint32_t *d_topbits, std::string &err);

// Bins a host matrix row by row.  out_mode 0: uint8 [n][p] ids clamped to
// bin_count - 1 into device memory `out` (the predict input), an id of 256
// stored as 255 with the row's bit set in d_topbits [d_bigidx[j]][ceil(n /
// 32)] (zeroed by the caller); 1: the raw uint16 [n][p] ids of
// _bin_features (E:2144-2189) into host memory `out`.
int bin_rows(Work *w, gbmh2d::Stager *sg, cudaStream_t st, const void *X, int64_t n, int p, int dtype,
             const double *edges, int stride, const int32_t *counts, const int32_t *nan_bin, int out_mode,
             void *out, const int32_t *d_bigidx, uint32_t *d_topbits, std::string &err);

}  // namespace gbmbin
