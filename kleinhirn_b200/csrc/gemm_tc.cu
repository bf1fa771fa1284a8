// tcgen05 GEMM of the encoder's projections: C = epilogue(A W^T + bias), A [M, K] f16 row-major
// (the activations), W [N, K] f16 row-major (PyTorch [out, in] weights, as the reference stores
// them, src/convert/names.ts:5), f32 accumulation in TMEM.
//
// Tiles are 128 x BN with BN = 256 when N is a multiple of 256 (the operands of one N = 256 MMA
// step stay within the shared-memory bandwidth of the SM), else BN = 128.
// One persistent CTA per SM, 320 threads in three roles:
//   warp 0      TMA producer: 128 x 64 tiles of A and BN x 64 tiles of W into a ring of STAGES
//               shared-memory stages (128-byte swizzle), completion on per-stage mbarriers;
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16 (M 128, N BN, K 16) into
//               one of two TMEM accumulators, commits each stage back to the producer and each
//               finished tile to the epilogue;
//   warps 2-9   epilogue, two warpgroups: warpgroup g takes accumulator columns
//               [g BN / 2, (g + 1) BN / 2) (warp w reads TMEM lanes 32 (w % 4) ..); bias, activation and the fused
//               follow-up op in registers, the f16 result into a swizzled shared-memory tile,
//               written out by one TMA store per warpgroup (rows and columns past M and N are
//               clipped by the tensor map).
// Tiles run n-fastest so the CTAs working at the same time share rows of A in L2.
//
// Epilogues reproduce the reference's storage rounding exactly (every value the reference
// stores in the plan's f16 buffer is rounded to f16 here before it is used again):
//   plain     C = f16(act(acc + bias))                              (matmul.wgsl / mmtile.wgsl)
//   residual  C = f16(C + f16(acc + bias))                          (matmul, then add.wgsl)
//   geglu     W rows interleaved per 64: C[r, j] = f16(gelu(f16(a + ba)) * f16(b + bb))
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
constexpr int BK = 64;
constexpr int A_BYTES = BM * BK * 2;
constexpr int OUT_BYTES = 128 * 64 * 2;  // one warpgroup's staged output tile
constexpr int THREADS = 320;
constexpr int EPI_THREADS = 256;

template <int BN>
struct GCfg {
  static constexpr int STAGES = BN == 256 ? 3 : 4;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + 4 * OUT_BYTES + 1024 + 256;
  static constexpr int WG_COLS = BN / 2;  // accumulator columns of one epilogue warpgroup
};

enum Epi { EPI_PLAIN = 0, EPI_RESIDUAL = 1, EPI_GEGLU = 2, EPI_ROPE = 3 };

struct Params {
  int M, N, K;
  const __half* bias;
  const __half* C;  // residual source (the output itself)
  int ldc;
  int act;
  int epi;
  const float* table;
  const int32_t* row_pos;
  int rope_cols;  // columns of q and k (2 H D), heads of 64
};

// GELU with the Abramowitz-Stegun 7.1.26 erf (the reference's formula and constants,
// src/kernels/mmtile.wgsl:22-31); the reciprocal and exp through the MUFU approximations, whose
// error is far below the f16 rounding of the stored result.
__device__ __forceinline__ float gelu_as(float v) {
  const float u = v * 0.7071067811865476f;
  const float t = rcp_approx(1.0f + 0.3275911f * fabsf(u));
  const float p = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                   0.254829592f) * t;
  const float e = 1.0f - p * ex2_approx(-(u * u) * 1.4426950408889634f);
  return 0.5f * v * (1.0f + (v >= 0.0f ? e : -e));
}

__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == 1) return fmaxf(v, 0.0f);
  if (act == 2) return gelu_as(v);
  if (act == 3) return tanhf(v);  // near 0 the exp form loses the relative precision f16 keeps
  if (act == 4) return v * rcp_approx(1.0f + ex2_approx(-v * 1.4426950408889634f));
  return v;
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

// 32 consecutive f16 values of a row (16-byte aligned) as f32
__device__ __forceinline__ void load32h(const __half* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = s[q];
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      v[q * 8 + 2 * e] = f.x;
      v[q * 8 + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void bias32(const __half* b, int n, float (&v)[32]) {
  if (b) {
    load32h(b + n, v);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
}

// Row r of a staged tile with 128-byte rows (128-byte swizzle, the TMA layout of a 64-column
// f16 box): the 16-byte chunks ch .. ch + 3 hold v[0 .. 31].
__device__ __forceinline__ void stage32_sw128(uint8_t* tile, int r, int ch, const float (&v)[32]) {
  uint8_t* row = tile + r * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
    *reinterpret_cast<uint4*>(row + (((ch + q) ^ (r & 7)) * 16)) = *reinterpret_cast<uint4*>(h);
  }
}

// Row r of a staged tile with 64-byte rows (64-byte swizzle, a 32-column f16 box).
__device__ __forceinline__ void stage32_sw64(uint8_t* tile, int r, const float (&v)[32]) {
  uint8_t* row = tile + r * 64;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
    *reinterpret_cast<uint4*>(row + ((q ^ ((r >> 1) & 3)) * 16)) = *reinterpret_cast<uint4*>(h);
  }
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const Params p) {
  using G = GCfg<BN>;
  constexpr int STAGES = G::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * G::B_BYTES;  // [warpgroup][2] 16 KB staging tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + 4 * OUT_BYTES);
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
      mbar_init(&tempty[b], EPI_THREADS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) tmem_alloc(tmem_holder, G::TMEM_COLS);
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
          mbar_arrive_expect_tx(&full[stage], A_BYTES + G::B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * G::B_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
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
          const uint64_t db = desc_sw128(sB + stage * G::B_BYTES);
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
    const int q = warp & 3;          // TMEM lane quarter of this warp
    const int g = (warp - 2) >> 2;   // warpgroup
    const int r = q * 32 + lane;     // row of the tile
    const bool leader = (warp == 2 + 4 * g) && lane == 0;
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
      const int row = mb * BM + r;
      const bool live = row < p.M;
      const int n0 = nb * BN;
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * BN);
      if (p.epi == EPI_GEGLU) {
        // accumulator columns [0, BN/2) hold a, [BN/2, BN) hold b for the tile's BN/2 outputs;
        // this warpgroup writes outputs [g OC, g OC + OC) of the tile
        constexpr int OC = BN / 4;
        uint8_t* stile = sOut + (g * 2 + buf) * OUT_BYTES;
        if (leader) bulk_wait_read<1>();
        named_bar(1 + g, 128);
#pragma unroll 1
        for (int pc = 0; pc < OC / 32; ++pc) {
          uint32_t ra[32], rb[32];
          tmem_ld32(taddr + g * OC + pc * 32, ra);
          tmem_ld32(taddr + BN / 2 + g * OC + pc * 32, rb);
          tmem_ld_wait();
          if (pc == OC / 32 - 1) {
            fence_before_sync();
            mbar_arrive(&tempty[buf]);  // the accumulator is read: the MMA may reuse it
          }
          float ba[32], bb[32], v[32];
          bias32(p.bias, n0 + g * OC + pc * 32, ba);
          bias32(p.bias, n0 + BN / 2 + g * OC + pc * 32, bb);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float a = f16r(__uint_as_float(ra[i]) + ba[i]);
            const float b = f16r(__uint_as_float(rb[i]) + bb[i]);
            v[i] = gelu_as(a) * b;
          }
          if (OC == 32) stage32_sw64(stile, r, v);
          else stage32_sw128(stile, r, pc * 4, v);
        }
        fence_proxy_async_smem();
        named_bar(1 + g, 128);
        if (leader) {
          tma_store_2d(&tmC, stile, nb * (BN / 2) + g * OC, mb * BM);
          bulk_commit();
        }
      } else {
#pragma unroll 1
        for (int ch = 0; ch < G::WG_COLS / 64; ++ch) {
          const int nc = n0 + g * G::WG_COLS + ch * 64;
          uint8_t* stile = sOut + (g * 2 + (BN == 128 ? buf : ch)) * OUT_BYTES;
          uint32_t r0[32], r1[32];
          tmem_ld32(taddr + g * G::WG_COLS + ch * 64, r0);
          tmem_ld32(taddr + g * G::WG_COLS + ch * 64 + 32, r1);
          tmem_ld_wait();
          if (ch == G::WG_COLS / 64 - 1) {
            fence_before_sync();
            mbar_arrive(&tempty[buf]);  // the accumulator is read: the MMA may reuse it
          }
          // the TMA store that last read this staging tile must be done with it
          if (leader) bulk_wait_read<1>();
          named_bar(1 + g, 128);
          float v0[32], v1[32];
          bias32(p.bias, min(nc, p.N - 32), v0);
          bias32(p.bias, min(nc + 32, p.N - 32), v1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v0[i] += __uint_as_float(r0[i]);
            v1[i] += __uint_as_float(r1[i]);
          }
          if (p.epi == EPI_ROPE && nc < p.rope_cols) {
            // one 64-wide head: rotate-half with the table row of the local position
            const float* tb = p.table + int64_t(live ? p.row_pos[row] : 0) * 128;
#pragma unroll
            for (int d = 0; d < 32; ++d) {
              const float x = f16r(v0[d]), y = f16r(v1[d]);
              const float cs = tb[d], sn = tb[64 + d];
              v0[d] = x * cs - y * sn;
              v1[d] = y * cs + x * sn;
            }
          } else if (p.epi == EPI_RESIDUAL) {
            float res[32];
            if (live && nc < p.N) {
              load32h(p.C + int64_t(row) * p.ldc + nc, res);
#pragma unroll
              for (int i = 0; i < 32; ++i) v0[i] = res[i] + f16r(v0[i]);
            }
            if (live && nc + 32 < p.N) {
              load32h(p.C + int64_t(row) * p.ldc + nc + 32, res);
#pragma unroll
              for (int i = 0; i < 32; ++i) v1[i] = res[i] + f16r(v1[i]);
            }
          } else if (p.act) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v0[i] = act_fn(v0[i], p.act);
              v1[i] = act_fn(v1[i], p.act);
            }
          }
          stage32_sw128(stile, r, 0, v0);
          stage32_sw128(stile, r, 4, v1);
          fence_proxy_async_smem();
          named_bar(1 + g, 128);
          if (leader) {
            if (nc < p.N) tma_store_2d(&tmC, stile, nc, mb * BM);
            bulk_commit();
          }
        }
      }
    }
    if (leader) bulk_wait<0>();
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    fence_after_sync();
    tmem_free(tmem, G::TMEM_COLS);
  }
}

}  // namespace

bool gemm_tc_supported(int N, int K) { return N >= 64 && N % 64 == 0 && K % 8 == 0 && K >= 16; }
bool gemm_tc_supported_geglu(int N, int K) { return N % 128 == 0 && gemm_tc_supported(N, K); }
bool gemm_tc_supported_rope(int D) { return D == 64; }

// Tile width of a GEMM with N outputs.
static int tile_n(int N) { return N % 256 == 0 ? 256 : 128; }

int gemm_geglu_group(int N) { return tile_n(N) / 2; }

// GeGLU input projection [2I, K] -> rows interleaved per G = gemm_geglu_group(N): block b holds
// rows [G b, G b + G) of the first half, then the same rows of the second half.
DevTensor gemm_geglu_weight(Ctx* ctx, const std::string& name, int N, int K) {
  const DevTensor& w = ctx->weight(name, true);
  DevTensor d;
  d.name = name + "#geglu-interleave";
  d.dtype = 1;
  d.shape = w.shape;
  d.bytes = size_t(N) * K * 2;
  KH_CUDA(cudaMalloc(&d.ptr, d.bytes));
  const int I = N / 2, G = gemm_geglu_group(N);
  const size_t row = size_t(K) * 2;
  for (int b = 0; b < I / G; ++b) {
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b) * G * row, (const char*)w.ptr + size_t(b) * G * row,
                            G * row, cudaMemcpyDeviceToDevice, ctx->stream));
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b + 1) * G * row,
                            (const char*)w.ptr + (size_t(I) + size_t(b) * G) * row, G * row,
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
  const int I = N / 2, G = gemm_geglu_group(N);
  for (int b = 0; b < I / G; ++b) {
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b) * G * 2, (const char*)w.ptr + size_t(b) * G * 2, G * 2,
                            cudaMemcpyDeviceToDevice, ctx->stream));
    KH_CUDA(cudaMemcpyAsync((char*)d.ptr + size_t(2 * b + 1) * G * 2, (const char*)w.ptr + size_t(I + b * G) * 2,
                            G * 2, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  KH_CUDA(cudaStreamSynchronize(ctx->stream));
  return d;
}

template <int BN>
static void launch_bn(const void* A, const void* W, void* C, const Params& p, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    KH_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, GCfg<BN>::SMEM));
    configured = true;
  }
  const int M = p.M, N = p.N, K = p.K;
  const CUtensorMap& ma = tensor_map_f16(A, uint64_t(M), uint64_t(K), uint64_t(K), BK, BM, 128);
  const CUtensorMap& mb = tensor_map_f16(W, uint64_t(N), uint64_t(K), uint64_t(K), BK, BN, 128);
  // output boxes: 64 columns (128-byte rows); GeGLU writes BN / 4 columns per warpgroup
  const CUtensorMap& mc =
      p.epi == EPI_GEGLU
          ? tensor_map_f16(C, uint64_t(M), uint64_t(N / 2), uint64_t(N / 2), BN / 4, 128, BN / 4 * 2)
          : tensor_map_f16(C, uint64_t(M), uint64_t(N), uint64_t(N), 64, 128, 128);
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  static const int sms = device_sms();
  const int grid = std::min(tiles, sms);
  gemm_tc_kernel<BN><<<grid, THREADS, GCfg<BN>::SMEM, st>>>(ma, mb, mc, p);
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
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.bias = static_cast<const __half*>(bias);
  p.C = static_cast<const __half*>(C);
  p.ldc = N;
  p.act = act;
  p.epi = EPI_PLAIN;
  p.table = nullptr;
  p.row_pos = nullptr;
  p.rope_cols = 0;
  if (e.kind == GemmEpilogue::Residual) {
    p.epi = EPI_RESIDUAL;
    if (act) throw PlanError("residual epilogue after an activation");
  } else if (e.kind == GemmEpilogue::GeGLU) {
    p.epi = EPI_GEGLU;
    p.ldc = N / 2;
  } else if (e.kind == GemmEpilogue::Rope) {
    if (e.D != 64) throw PlanError("rope epilogue needs 64-wide heads");
    p.epi = EPI_ROPE;
    p.table = e.table;
    p.row_pos = e.row_pos;
    p.rope_cols = 2 * e.H * e.D;
  }
  if (tile_n(N) == 256) launch_bn<256>(A, W, C, p, st);
  else launch_bn<128>(A, W, C, p, st);
}

int tc_error_code() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sm100::kh_tc_error, sizeof(int));
  return v;
}

}  // namespace kh
