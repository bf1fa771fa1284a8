// TMA tensor maps of row-major f16 matrices (host side), cached by shape and pointer.
#pragma once

#include <atomic>
#include <cstdint>
#include <functional>

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

// Runs `configure` once per device (the current one) and process: kernel attributes such as the
// shared-memory limit are per device, and several contexts of one process may drive different
// devices from different host threads.
void once_per_device(std::atomic<uint64_t>& done, const std::function<void()>& configure);

}  // namespace kh
