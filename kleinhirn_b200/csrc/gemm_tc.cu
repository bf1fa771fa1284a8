// tcgen05 GEMM of the encoder's projections: C = epilogue(A W^T + bias), A [M, K] f16 row-major
// (the activations), W [N, K] f16 row-major (PyTorch [out, in] weights, as the reference stores
// them, src/convert/names.ts:5), f32 accumulation in TMEM.
//
// One persistent CTA per SM, 192 threads in three roles:
//   warp 0      TMA producer: 128 x 64 tiles of A and BN x 64 tiles of W into a ring of STAGES
//               shared-memory stages (128-byte swizzle), completion on per-stage mbarriers;
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16 (M 128, N BN, K 16) into
//               one of two TMEM accumulators, commits each stage back to the producer and each
//               finished tile to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32 (w % 4) ..),
//               bias, activation and the fused follow-up op, f16 store.
// Tiles run n-fastest so the CTAs working at the same time share rows of A in L2.
//
// Epilogues reproduce the reference's storage rounding exactly (every value the reference
// stores in the plan's f16 buffer is rounded to f16 here before it is used again):
//   plain     C = f16(act(acc + bias))                              (matmul.wgsl / mmtile.wgsl)
//   residual  C = f16(C + f16(acc + bias))                          (matmul, then add.wgsl)
//   geglu     W rows interleaved per 64 columns: C[r, j] = f16(gelu(f16(a + ba)) * f16(b + bb))
//                                                                   (matmul, then geglu.wgsl)
//   rope      q and k head blocks rotated with the f32 cos / sin table row of the local position:
//             C = f16(x c - y s), f16(y c + x s) with x, y = f16(acc + bias) (matmul, then rope.wgsl)

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "gemm_tc.h"
#include "sm100.cuh"
#include "tmap.h"

namespace kh {

namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + 1024 + 256;

enum Epi { EPI_PLAIN = 0, EPI_RESIDUAL = 1, EPI_GEGLU = 2, EPI_ROPE = 3 };

struct Params {
  int M, N, K;
  const __half* bias;
  __half* C;
  int ldc;
  int act;
  int epi;
  const float* table;
  const int32_t* row_pos;
  int D;          // rope head dimension
  int rope_cols;  // columns of q and k (2 H D)
};

__device__ __forceinline__ float gelu_as(float v) {
  const float u = v * 0.7071067811865476f;
  const float t = 1.0f / (1.0f + 0.3275911f * fabsf(u));
  const float p = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                   0.254829592f) * t;
  const float e = 1.0f - p * expf(-u * u);
  return 0.5f * v * (1.0f + (v >= 0.0f ? e : -e));
}

__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == 1) return fmaxf(v, 0.0f);
  if (act == 2) return gelu_as(v);
  if (act == 3) return tanhf(v);
  if (act == 4) return v / (1.0f + expf(-v));
  return v;
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ void store32(__half* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
    d[q] = *reinterpret_cast<uint4*>(h);
  }
}

__device__ __forceinline__ void load32(const __half* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u = s[q];
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __half22float2(h[e]);
      v[q * 8 + 2 * e] = f.x;
      v[q * 8 + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float bias_at(const __half* b, int n) { return b ? __half2float(b[n]) : 0.0f; }

__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (p.M + BM - 1) / BM, n_tiles = (p.N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;  // stages with a load issued, parity of their last load
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mb = t / n_tiles, nb = t % n_tiles;
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        // let every copy this thread issued land before the CTA ends
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&full[s], (last_parity >> s) & 1u, 11);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[buf], tphase ^ 1, 2)) {
          ok = false;
          break;
        }
        fence_after_sync();
        const uint32_t d = tmem + uint32_t(buf * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, 3)) {
            ok = false;
            break;
          }
          fence_after_sync();
          const uint64_t da = desc_sw128(sA + stage * A_BYTES);
          const uint64_t db = desc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16(d, da + uint64_t(k * 2), db + uint64_t(k * 2), idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);
      }
      if (!ok) {
        *abort_flag = 1;
        mma_commit(drain);  // wait for the MMAs in flight before the TMEM is freed
        mbar_wait(drain, 0, 12);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter of this warp
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      if (*abort_flag || !mbar_wait(&tfull[buf], tphase, 4)) {
        *abort_flag = 1;
        break;
      }
      fence_after_sync();
      const int mb = t / n_tiles, nb = t % n_tiles;
      const int row = mb * BM + q * 32 + lane;
      const bool live = row < p.M;
      const int n0 = nb * BN;
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * BN);
      if (p.epi == EPI_GEGLU) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t ra[32], rb[32];
          tmem_ld32(taddr + c * 32, ra);
          tmem_ld32(taddr + 64 + c * 32, rb);
          tmem_ld_wait();
          const int g0 = nb * 64 + c * 32;
          if (live && g0 < p.ldc) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float a = f16r(__uint_as_float(ra[i]) + bias_at(p.bias, n0 + c * 32 + i));
              const float b = f16r(__uint_as_float(rb[i]) + bias_at(p.bias, n0 + 64 + c * 32 + i));
              v[i] = gelu_as(a) * b;
            }
            store32(p.C + int64_t(row) * p.ldc + g0, v);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          uint32_t r0[32], r1[32];
          tmem_ld32(taddr + c * 32, r0);
          tmem_ld32(taddr + (c + 1) * 32, r1);
          tmem_ld_wait();
          const int n = n0 + c * 32;
          if (!live || n >= p.N) continue;
          float v[64];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = __uint_as_float(r0[i]) + bias_at(p.bias, n + i);
            v[32 + i] = __uint_as_float(r1[i]) + bias_at(p.bias, n + 32 + i);
          }
          __half* dst = p.C + int64_t(row) * p.ldc + n;
          if (p.epi == EPI_ROPE && n < p.rope_cols) {
            // one 64-wide head (D == 64): rotate-half with the table row of the local position
            const float* tb = p.table + int64_t(p.row_pos[row]) * 2 * 64;
#pragma unroll
            for (int d = 0; d < 32; ++d) {
              const float x = f16r(v[d]), y = f16r(v[d + 32]);
              const float cs = tb[d], sn = tb[64 + d];
              v[d] = x * cs - y * sn;
              v[d + 32] = y * cs + x * sn;
            }
          } else if (p.epi == EPI_RESIDUAL) {
            float r[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              load32(dst + h * 32, r);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[h * 32 + i] = r[i] + f16r(v[h * 32 + i]);
            }
          } else if (p.act) {
#pragma unroll
            for (int i = 0; i < 64; ++i) v[i] = act_fn(v[i], p.act);
          }
          float lo[32], hi[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            lo[i] = v[i];
            hi[i] = v[32 + i];
          }
          store32(dst, lo);
          if (n + 32 < p.N) store32(dst + 32, hi);
        }
      }
      fence_before_sync();
      mbar_arrive(&tempty[buf]);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    fence_after_sync();
    tmem_free(tmem, TMEM_COLS);
  }
}

}  // namespace

bool gemm_tc_supported(int N, int K) { return N >= 32 && N % 32 == 0 && K % 8 == 0 && K >= 16; }
bool gemm_tc_supported_geglu(int N, int K) { return N % 128 == 0 && gemm_tc_supported(N, K); }
bool gemm_tc_supported_rope(int D) { return D == 64; }

// GeGLU input projection [2I, K] -> rows interleaved per 64: block b holds rows [64 b, 64 b + 64)
// of the first half, then the same rows of the second half.
DevTensor gemm_geglu_weight(Ctx* ctx, const std::string& name, int N, int K) {
  const DevTensor& w = ctx->weight(name, true);
  DevTensor d;
  d.name = name + "#geglu-interleave";
  d.dtype = 1;
  d.shape = w.shape;
  d.bytes = size_t(N) * K * 2;
  KH_CUDA(cudaMalloc(&d.ptr, d.bytes));
  const int I = N / 2;
  const size_t row = size_t(K) * 2;
  for (int b = 0; b < I / 64; ++b) {
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b) * 64 * row, (const char*)w.ptr + size_t(b) * 64 * row,
                            64 * row, cudaMemcpyDeviceToDevice, ctx->stream));
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b + 1) * 64 * row,
                            (const char*)w.ptr + (size_t(I) + size_t(b) * 64) * row, 64 * row,
                            cudaMemcpyDeviceToDevice, ctx->stream));
  }
  KH_CUDA(cudaStreamSynchronize(ctx->stream));
  return d;
}

DevTensor gemm_geglu_bias(Ctx* ctx, const std::string& name, int N) {
  const DevTensor& w = ctx->weight(name, true);
  DevTensor d;
  d.name = name + "#geglu-interleave";
  d.dtype = 1;
  d.shape = w.shape;
  d.bytes = size_t(N) * 2;
  KH_CUDA(cudaMalloc(&d.ptr, d.bytes));
  const int I = N / 2;
  for (int b = 0; b < I / 64; ++b) {
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b) * 128, (const char*)w.ptr + size_t(b) * 128, 128,
                            cudaMemcpyDeviceToDevice, ctx->stream));
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b + 1) * 128, (const char*)w.ptr + size_t(I + b * 64) * 2, 128,
                            cudaMemcpyDeviceToDevice, ctx->stream));
  }
  KH_CUDA(cudaStreamSynchronize(ctx->stream));
  return d;
}

void launch_gemm(Ctx* ctx, bool f16, const void* A, const void* W, const void* bias, void* C, int M, int N, int K,
                 int act, const GemmEpilogue& e, cudaStream_t st) {
  (void)ctx;
  if (M <= 0) return;
  if (!f16 || !gemm_tc_supported(N, K)) {
    if (e.kind != GemmEpilogue::None) throw PlanError("gemm epilogue without the tensor-core path");
    launch_gemm_simt(f16, A, W, bias, C, M, N, K, act, st);
    return;
  }
  static bool configured = false;
  if (!configured) {
    KH_CUDA(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured = true;
  }
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.bias = static_cast<const __half*>(bias);
  p.C = static_cast<__half*>(C);
  p.ldc = N;
  p.act = act;
  p.epi = EPI_PLAIN;
  p.table = nullptr;
  p.row_pos = nullptr;
  p.D = 0;
  p.rope_cols = 0;
  if (e.kind == GemmEpilogue::Residual) {
    p.epi = EPI_RESIDUAL;
    if (act) throw PlanError("residual epilogue after an activation");
  } else if (e.kind == GemmEpilogue::GeGLU) {
    p.epi = EPI_GEGLU;
    p.ldc = N / 2;
  } else if (e.kind == GemmEpilogue::Rope) {
    p.epi = EPI_ROPE;
    p.table = e.table;
    p.row_pos = e.row_pos;
    p.D = e.D;
    p.rope_cols = 2 * e.H * e.D;
  }
  const CUtensorMap& ma = tensor_map_f16(A, uint64_t(M), uint64_t(K), uint64_t(K), BK, BM, 128);
  const CUtensorMap& mb = tensor_map_f16(W, uint64_t(N), uint64_t(K), uint64_t(K), BK, BN, 128);
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  static const int sms = device_sms();
  const int grid = std::min(tiles, sms);
  gemm_tc_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(ma, mb, p);
}

int tc_error_code() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sm100::kh_tc_error, sizeof(int));
  return v;
}

}  // namespace kh
