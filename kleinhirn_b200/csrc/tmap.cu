// TMA tensor-map encoding through the driver entry point, cached per (pointer, geometry).

#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "runtime.h"
#include "tmap.h"

namespace kh {

namespace {

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  if (!fn) throw CudaError("cuTensorMapEncodeTiled is unavailable");
  return fn;
}

}  // namespace

namespace {
void encode_2d(CUtensorMap* out, CUtensorMapDataType dtype, uint64_t esize, const void* ptr, uint64_t rows,
               uint64_t cols, uint64_t row_stride, uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (row_stride * esize) % 16)
    throw PlanError("tensor map: base or row stride not 16-byte aligned");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride * esize};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  const CUresult r = encode_fn()(out, dtype, 2, const_cast<void*>(ptr), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
}
}  // namespace

void encode_tensor_map_f16(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride,
                           uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  encode_2d(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptr, rows, cols, row_stride, box_cols, box_rows, swizzle_bytes);
}

CUtensorMap tensor_map_f32(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_cols,
                           uint32_t box_rows) {
  // (f32 operands of the 3xTF32 GEMM: 128-byte swizzle; cached and copied out like the f16 maps)
  static std::mutex mu;
  static std::map<std::tuple<const void*, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(ptr, rows, cols, row_stride, box_cols, box_rows);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cache.size() > 8192) cache.clear();
  CUtensorMap m;
  encode_2d(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ptr, rows, cols, row_stride, box_cols, box_rows, 128);
  cache.emplace(key, m);
  return m;
}

CUtensorMap tensor_map_f16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_cols,
                           uint32_t box_rows, int swizzle_bytes) {
  // The map is copied out while the lock is held: another host thread (a context on another
  // device) may clear the cache at any time after the lock is released.
  static std::mutex mu;
  static std::map<std::tuple<const void*, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(ptr, rows, cols, row_stride, box_cols, box_rows, swizzle_bytes);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cache.size() > 8192) cache.clear();
  CUtensorMap m;
  encode_tensor_map_f16(&m, ptr, rows, cols, row_stride, box_cols, box_rows, swizzle_bytes);
  cache.emplace(key, m);
  return m;
}

int64_t selftest_tensor_maps(int threads, int iters) {
  // Threads fetch maps of distinct (pointer, geometry) keys, more than the cache keeps, so the
  // cache is cleared while others hold their copies; every copy must equal a fresh encoding.
  if (threads < 1 || threads > 64 || iters < 1 || iters > 100000)
    throw ArgError("tensor-map self-test: threads in [1, 64], iters in [1, 1e5]");
  void* base = nullptr;
  KH_CUDA(cudaMalloc(&base, size_t(1) << 20));
  std::atomic<int64_t> bad{0};
  std::vector<std::thread> pool;
  std::vector<std::string> errs(static_cast<size_t>(threads));
  int dev = current_device();
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&, t] {
      try {
        KH_CUDA(cudaSetDevice(dev));
        for (int i = 0; i < iters; ++i) {
          const uint64_t off = uint64_t((t * 7919 + i * 104729) % 65000) * 16;
          const char* p = static_cast<const char*>(base) + off;
          const uint64_t rows = 64 + uint64_t((i + t) % 5);
          const CUtensorMap m = tensor_map_f16(p, rows, 64, 64, 64, 64, 128);
          CUtensorMap fresh;
          encode_tensor_map_f16(&fresh, p, rows, 64, 64, 64, 64, 128);
          if (std::memcmp(&m, &fresh, sizeof(CUtensorMap)) != 0) bad.fetch_add(1);
        }
      } catch (const std::exception& e) {
        errs[size_t(t)] = e.what();
      }
    });
  for (auto& th : pool) th.join();
  cudaFree(base);
  for (const auto& e : errs)
    if (!e.empty()) throw CudaError("tensor-map self-test: " + e);
  return bad.load();
}

void once_per_device(std::atomic<uint64_t>& done, const std::function<void()>& configure) {
  int dev = 0;
  KH_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw ArgError("device ordinal above 63");
  const uint64_t bit = 1ull << dev;
  if (done.load(std::memory_order_acquire) & bit) return;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (done.load(std::memory_order_relaxed) & bit) return;
  configure();
  done.fetch_or(bit, std::memory_order_release);
}

int device_sms() {
  // SM count of the current device, looked up once per device (contexts of one process may drive
  // devices with different counts from different host threads)
  static std::atomic<int> sms_of[64] = {};
  int dev = 0;
  KH_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw ArgError("device ordinal above 63");
  int sms = sms_of[dev].load(std::memory_order_relaxed);
  if (sms <= 0) {
    KH_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    sms_of[dev].store(sms, std::memory_order_relaxed);
  }
  return sms;
}

int current_device() {
  int dev = 0;
  KH_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw ArgError("device ordinal above 63");
  return dev;
}

}  // namespace kh
