// tmap.cuh — host-side TMA tensor-map construction for 2-D uint8 tensors.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace mfi {

// 2-D uint8 tensor of `rows` rows of `row_bytes` bytes (row stride = row_bytes),
// box 128 bytes x box_rows, 128-byte swizzle, zero fill outside the tensor.
bool make_tmap(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
               uint32_t box_rows);

// Same, memoised on (base, row_bytes, rows, box_rows): weight and workspace
// maps are reused across calls without re-encoding.
bool get_tmap(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
              uint32_t box_rows);

// Unswizzled map with a box of box_bytes (a multiple of 16) x box_rows,
// memoised like get_tmap.
bool get_tmap_plain(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
                    uint32_t box_bytes, uint32_t box_rows);

// Grant kernel `fn` `bytes` of dynamic shared memory on the current device
// (cudaFuncSetAttribute once per device and size; thread-safe).
cudaError_t ensure_dynamic_smem(const void* fn, size_t bytes);

}  // namespace mfi
