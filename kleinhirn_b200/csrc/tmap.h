// TMA tensor maps of row-major f16 matrices (host side), cached by shape and pointer.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace kh {

// Map of a row-major f16 matrix of `rows` x `cols` with rows `row_stride` elements apart; tiles
// of box_cols x box_rows elements, swizzle 128 / 64 / 32 bytes (or none), zero fill outside.
const CUtensorMap& tensor_map_f16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride,
                                  uint32_t box_cols, uint32_t box_rows, int swizzle_bytes);

// The same map encoded into `out`, without the cache.
void encode_tensor_map_f16(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride,
                           uint32_t box_cols, uint32_t box_rows, int swizzle_bytes);

int device_sms();

}  // namespace kh
