// TMA tensor maps of row-major f16 matrices (host side), cached by shape and pointer.
#pragma once

#include <atomic>
#include <cstdint>
#include <functional>

#include <cuda.h>

namespace kh {

// Map of a row-major f16 matrix of `rows` x `cols` with rows `row_stride` elements apart; tiles
// of box_cols x box_rows elements, swizzle 128 / 64 / 32 bytes (or none), zero fill outside.
// Encoded once per (pointer, geometry) and cached; returned by value, so a caller's copy stays
// valid whatever other threads do to the cache.
CUtensorMap tensor_map_f16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_cols,
                           uint32_t box_rows, int swizzle_bytes);

// Map of a row-major f32 matrix (128-byte swizzle, zero fill outside), cached like the f16 maps.
CUtensorMap tensor_map_f32(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_cols,
                           uint32_t box_rows);

// The f16 map encoded into `out`, without the cache.
void encode_tensor_map_f16(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride,
                           uint32_t box_cols, uint32_t box_rows, int swizzle_bytes);

// Self-test of the cache under concurrent use: `threads` host threads fetch `iters` maps each over
// more keys than the cache keeps; returns how many fetched maps differ from a fresh encoding.
int64_t selftest_tensor_maps(int threads, int iters);

// SM count of the current device (looked up once per device).
int device_sms();

// Ordinal of the current device, checked to lie in [0, 64).
int current_device();

// Runs `configure` once per device (the current one) and process: kernel attributes such as the
// shared-memory limit are per device, and several contexts of one process may drive different
// devices from different host threads.
void once_per_device(std::atomic<uint64_t>& done, const std::function<void()>& configure);

}  // namespace kh
