// h2d.h -- host -> device streaming of row-major host arrays through a ring
// of pinned buffers.
//
// Host worker threads copy (or narrow) each chunk of rows into a pinned
// buffer while the chunks before it are still being copied to the device,
// so a large upload runs at the DMA rate rather than at the rate of the
// driver's single-threaded staging of pageable memory.  A chunk's consumer
// (typically a kernel that transposes or bins the rows) is enqueued on the
// same stream right after the chunk's copy.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace gbmh2d {

enum class Pack {
    Copy,      // rows are copied as they are
    U16toU8,   // uint16 -> uint8 as min(v, 255); values above 255 are listed in `wide`
};

struct Stager;

Stager *stager_create();
void stager_destroy(Stager *s);

// Streams `rows` rows of `row_bytes` host bytes each (packed bytes per row:
// row_bytes, or row_bytes / 2 for U16toU8).  For every chunk of rows
// [r0, r0 + nr) the packed rows are copied to dst(r0, nr) on `st`; then
// after(r0, nr, that address) enqueues the chunk's consumer (it returns 0 or
// an error, with `err` set).  `max_chunk_rows` (> 0) bounds a chunk, e.g.
// to the size of a device staging buffer.  Returns 0, or -1 with `err` set.
// When it returns 0 all host reads of `src` are complete; device work may
// still be in flight on `st`.
// With U16toU8 and `wide` given, the element index (row * p + feature of
// the uint16 matrix) of every value above 255 is appended to *wide.
int stream_rows(Stager *s, cudaStream_t st, const void *src, int64_t rows, size_t row_bytes, Pack pack,
                int64_t max_chunk_rows, const std::function<void *(int64_t r0, int64_t nr)> &dst,
                const std::function<int(int64_t r0, int64_t nr, const void *dev)> &after, std::string &err,
                std::vector<int64_t> *wide = nullptr);

// Bytes a chunk may hold (the pinned buffer size).
size_t chunk_bytes();

}  // namespace gbmh2d
