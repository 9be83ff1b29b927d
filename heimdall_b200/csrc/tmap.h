#pragma once
#include <cuda.h>
#include <stdint.h>

namespace bfb {
// rank-N tiled map with optional 128-byte swizzle (dims/box innermost first, strides in bytes for dims 1..N-1)
int make_tmap(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);
// K-major 16-bit operand [rows][K] (row stride ld elements) loaded as (box_rows x 64*atoms) SW128 tiles
int make_tmap_kmajor(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t K, uint64_t ld,
                     uint32_t box_rows, uint32_t atoms);
}  // namespace bfb
