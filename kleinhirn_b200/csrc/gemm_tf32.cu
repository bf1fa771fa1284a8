// tcgen05 GEMM of f32 plans: C = act(A W^T + bias) in f32 through the 3xTF32 split.
//
// The tensor cores multiply TF32 values (10-bit mantissas) with f32 accumulation. Splitting each
// f32 operand as x = hi + lo, hi the TF32 value of x's leading bits and lo = x - hi (exact),
// A W^T = A_hi W_hi + A_hi W_lo + A_lo W_hi + A_lo W_lo, and the last term is below f32
// precision; the three others run as three kind::tf32 MMAs per K step into one accumulator. This
// is the published error-compensated TF32 method (three TF32 products recovering f32 accuracy);
// the result matches an f32 GEMM to about 2^-21 relative per product, the accuracy f32 plans ask
// for (the reference's WASM executor computes them in f32).
//
// Tiles are 128 x 64 (one M = 128 MMA per CTA, the accumulator in 64 TMEM columns), one per CTA:
//   warp 0     TMA: 32-column (128-byte) K slices of A (f32), W_hi and W_lo per stage into a
//              four-stage ring (128-byte swizzle);
//   warps 2-5  first split each stage's A into A_hi (in place) and A_lo (the stage's second A
//              slot), then, once the accumulator is done, the epilogue: each thread one
//              accumulator row (TMEM lane), bias and activation in f32 (the CUDA-core kernels'
//              arithmetic), stored to C;
//   warp 1     one thread issues, per 8-wide K step, A_lo W_hi, A_hi W_lo and A_hi W_hi.
// Launches of few tiles (short calls) split K: the grid's z splits of a tile form one cluster,
// each CTA accumulates its K blocks and writes the partial tile to its shared memory, and CTA z
// then sums rows [z R, (z + 1) R) of all partials in split order over distributed shared memory
// (deterministic), adds bias and activation and stores them.
// Rows, columns and K past the matrices are zero-filled by the tensor maps and not stored.

#include <algorithm>
#include <atomic>
#include <string>

#include "act_f32.cuh"
#include "gemm_tf32.h"
#include "sm100.cuh"
#include "tmap.h"

namespace kh {

namespace {

using namespace sm100;

constexpr int XBM = 128;                 // rows of a tile (one M = 128 MMA)
constexpr int XBN = 64;                  // columns of a tile (accumulator columns)
constexpr int XBK = 32;                  // K per stage: 32 f32 = 128-byte rows, the swizzle width
constexpr int XA = XBM * XBK * 4;        // 16 KB
constexpr int XB = XBN * XBK * 4;        // 8 KB
constexpr int XSTAGE = 2 * XA + 2 * XB;  // A_hi, A_lo, W_hi, W_lo: 48 KB
constexpr int XSTAGES = 4;
constexpr int XTHREADS = 64 + 128;       // producer warp, MMA warp, four epilogue warps
constexpr int XSMEM = XSTAGES * XSTAGE + 1024 + 256;

// kind::tf32 instruction descriptor: TF32 A and B (format 2), f32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}

__global__ void tf32_split_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float v = x[i];
    const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);  // sign, exponent, 10 mantissa bits
    hi[i] = h;
    lo[i] = v - h;
  }
}

struct XParams {
  int M, N, K, act;
  const float* bias;
  float* C;
  int kps;  // 32-wide K blocks per split (split-K launches: gridDim.z splits, one cluster)
};

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__global__ void __launch_bounds__(XTHREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmWh, const __grid_constant__ CUtensorMap tmWl,
                       const XParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + XSTAGES * XSTAGE);
  uint64_t* empty = full + XSTAGES;
  uint64_t* done = empty + XSTAGES;
  uint64_t* drain = done + 1;
  uint64_t* conv = drain + 1;  // [XSTAGES]: the stage's A split into hi and lo by the epilogue warps
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(conv + XSTAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * XBN, m0 = blockIdx.y * XBM;
  const int nk_all = (p.K + XBK - 1) / XBK;
  const bool splitk = gridDim.z > 1;
  // this CTA's K blocks [kb0, kb0 + nk): all of them, or split blockIdx.z of a split-K cluster
  const int kb0 = splitk ? int(blockIdx.z) * p.kps : 0;
  const int nk = splitk ? min(p.kps, nk_all - kb0) : nk_all;

  if (threadIdx.x == 0) {
    for (int s = 0; s < XSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 128);
    }
    mbar_init(done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmWh);
    prefetch_tmap(&tmWl);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 64);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      uint32_t issued = 0, parity = 0;  // stages with a load in flight, and the phase it completes
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % XSTAGES;
        const uint32_t u = uint32_t(kb / XSTAGES);
        if (*abort_flag || !mbar_wait(&empty[s], (u & 1) ^ 1, 81)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * XSTAGE;
        mbar_arrive_expect_tx(&full[s], XA + 2 * XB);  // A (f32), W_hi, W_lo
        const int kx = (kb0 + kb) * XBK;
        tma_load_2d(st, &tmA, &full[s], kx, m0);
        tma_load_2d(st + 2 * XA, &tmWh, &full[s], kx, n0);
        tma_load_2d(st + 2 * XA + XB, &tmWl, &full[s], kx, n0);
        issued |= 1u << s;
        parity = (parity & ~(1u << s)) | ((u & 1) << s);
      }
      if (!ok) {
        *abort_flag = 1;
        for (int s = 0; s < XSTAGES; ++s)  // every copy issued lands before the CTA ends
          if (issued & (1u << s)) mbar_wait(&full[s], (parity >> s) & 1u, 85);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(XBM, XBN);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % XSTAGES;
        const uint32_t u = uint32_t(kb / XSTAGES);
        if (*abort_flag || !mbar_wait(&conv[s], u & 1, 82)) {
          ok = false;
          break;
        }
        fence_after_sync();
        uint8_t* st = smem + s * XSTAGE;
        const uint64_t ah = desc_sw128(st), al = desc_sw128(st + XA);
        const uint64_t wh = desc_sw128(st + 2 * XA), wl = desc_sw128(st + 2 * XA + XB);
#pragma unroll
        for (int k = 0; k < XBK / 8; ++k) {  // 8 TF32 values = 32 bytes per MMA step
          const uint64_t o = uint64_t(2 * k);
          mma_tf32(tmem, al + o, wh + o, idesc, (kb | k) ? 1u : 0u);  // the small terms first
          mma_tf32(tmem, ah + o, wl + o, idesc, 1u);
          mma_tf32(tmem, ah + o, wh + o, idesc, 1u);
        }
        mma_commit(&empty[s]);
      }
      if (!ok) {
        *abort_flag = 1;
        mma_commit(drain);
        mbar_wait(drain, 0, 83);
      }
      mma_commit(done);  // (after a failure too: the epilogue then stores nothing)
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes 32 quarter .. : the rows this warp reads
    const int row = m0 + quarter * 32 + lane;
    // Until the accumulator is done these warps split each stage's A tile for the MMAs: hi (the
    // TF32 value of the leading bits) in place, lo = x - hi into the stage's second A slot, at the
    // same (swizzled) positions, so both tiles keep the tensor map's layout.
    const int ct = threadIdx.x - 64;  // 0 .. 127
    bool cok = true;
    for (int kb = 0; kb < nk && cok; ++kb) {
      const int s = kb % XSTAGES;
      const uint32_t u = uint32_t(kb / XSTAGES);
      cok = __all_sync(0xffffffffu, !*abort_flag && mbar_wait(&full[s], u & 1, 86));
      if (!cok) break;
      float4* a = reinterpret_cast<float4*>(smem + s * XSTAGE);
      float4* alo = reinterpret_cast<float4*>(smem + s * XSTAGE + XA);
#pragma unroll
      for (int i = 0; i < XA / 16 / 128; ++i) {
        const float4 v = a[ct + 128 * i];
        const float4 h = make_float4(__uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                                     __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                                     __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                                     __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
        a[ct + 128 * i] = h;
        alo[ct + 128 * i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      }
      fence_proxy_async_smem();  // the tensor core (async proxy) reads what these threads wrote
      mbar_arrive(&conv[s]);
    }
    if (!cok) *abort_flag = 1;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0, 84)) && !*abort_flag;
    fence_after_sync();
    const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16);
    float* part = reinterpret_cast<float*>(smem);  // split-K: [128][XBN + 1] over the stages (all read)
#pragma unroll 1
    for (int c0 = 0; c0 < XBN; c0 += 32) {
      uint32_t v[32];
      tmem_ld32(taddr + uint32_t(c0), v);
      tmem_ld_wait();
      if (splitk) {
        float* prow = part + (quarter * 32 + lane) * (XBN + 1) + c0;
#pragma unroll
        for (int i = 0; i < 32; ++i) prow[i] = __uint_as_float(v[i]);
        continue;
      }
      if (!ok || row >= p.M) continue;
      float* crow = p.C + int64_t(row) * p.N;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int col = n0 + c0 + i;
        if (col < p.N)
          crow[col] = f32act::activate(__uint_as_float(v[i]) + (p.bias ? p.bias[col] : 0.f), p.act);
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (splitk) {
    // C = sum of the splits' partials, in split order (deterministic), over distributed shared
    // memory: CTA z of the cluster reduces rows [z R, (z + 1) R) of the tile
    cluster_sync();
    const int S = int(gridDim.z), z = int(blockIdx.z);
    const int R = (XBM + S - 1) / S;
    const float* part = reinterpret_cast<const float*>(smem);
    for (int e = threadIdx.x; e < R * XBN; e += XTHREADS) {
      const int r = z * R + e / XBN, c = e % XBN;
      if (r >= XBM) break;
      const uint32_t a = smem_u32(part + r * (XBN + 1) + c);
      float acc = 0.f;
      for (int q = 0; q < S; ++q) {
        uint32_t aq;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(aq) : "r"(a), "r"(q));
        acc += ld_cluster_f32(aq);
      }
      const int grow = m0 + r, gcol = n0 + c;
      if (grow < p.M && gcol < p.N && !*abort_flag)
        p.C[int64_t(grow) * p.N + gcol] = f32act::activate(acc + (p.bias ? p.bias[gcol] : 0.f), p.act);
    }
    cluster_sync();  // no CTA leaves while another reads its partial
  }
  if (warp == 1) {
    fence_after_sync();
    tmem_free(tmem, 64);
  }
}

}  // namespace

bool gemm_tf32_supported(int N, int K) { return N >= 16 && K >= 4 && K % 4 == 0; }

void launch_tf32_split(const float* x, float* hi, float* lo, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  tf32_split_kernel<<<unsigned(blocks), 256, 0, st>>>(x, hi, lo, n);
  KH_CUDA(cudaGetLastError());
}

const DevTensor& gemm_tf32_weight(Ctx* ctx, const std::string& name) {
  return ctx->derive(name + "#tf32-split", [&]() {
    const DevTensor& w = ctx->weight(name, false);
    DevTensor d;
    d.name = name + "#tf32-split";
    d.dtype = 0;
    d.shape = w.shape;
    const int64_t n = w.numel();
    d.bytes = size_t(n) * 2 * 4;
    KH_CUDA(cudaMalloc(&d.ptr, d.bytes));
    float* hi = static_cast<float*>(d.ptr);
    launch_tf32_split(static_cast<const float*>(w.ptr), hi, hi + n, n, ctx->stream);
    KH_CUDA(cudaStreamSynchronize(ctx->stream));
    return d;
  });
}

void launch_gemm_tf32x3(const float* a, const float* w_hi, const float* w_lo, const float* bias, float* C, int M,
                        int N, int K, int act, cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  if (!gemm_tf32_supported(N, K)) throw PlanError("gemm (3xTF32): N < 16 or K not a multiple of 4");
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    KH_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, XSMEM));
  });
  const CUtensorMap ma = tensor_map_f32(a, uint64_t(M), uint64_t(K), uint64_t(K), XBK, XBM);
  const CUtensorMap mwh = tensor_map_f32(w_hi, uint64_t(N), uint64_t(K), uint64_t(K), XBK, XBN);
  const CUtensorMap mwl = tensor_map_f32(w_lo, uint64_t(N), uint64_t(K), uint64_t(K), XBK, XBN);
  XParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.act = act;
  p.bias = bias;
  p.C = C;
  const int tiles = ((N + XBN - 1) / XBN) * ((M + XBM - 1) / XBM);
  const int nk = (K + XBK - 1) / XBK;
  // Split-K for launches of few tiles (short calls): up to 8 splits of at least two K blocks each,
  // one cluster per tile, so that about every SM takes part
  int S = 1;
  if (tiles < 74) S = std::min({8, 148 / tiles, std::max(1, nk / 2)});
  p.kps = (nk + S - 1) / S;
  S = (nk + p.kps - 1) / p.kps;  // every split keeps at least one K block
  const dim3 grid(unsigned((N + XBN - 1) / XBN), unsigned((M + XBM - 1) / XBM), unsigned(S));
  if (S == 1) {
    gemm_tf32x3_kernel<<<grid, XTHREADS, XSMEM, st>>>(ma, mwh, mwl, p);
  } else {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = unsigned(S);
    cfg.gridDim = grid;
    cfg.blockDim = dim3(XTHREADS, 1, 1);
    cfg.dynamicSmemBytes = XSMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KH_CUDA(cudaLaunchKernelEx(&cfg, gemm_tf32x3_kernel, ma, mwh, mwl, p));
  }
  KH_CUDA(cudaGetLastError());
}

int tf32_error_code() {
  // read and cleared (after a sync of the work that may have set it)
  int v = 0;
  KH_CUDA(cudaMemcpyFromSymbol(&v, sm100::kh_tc_error, sizeof(int)));
  if (v) {
    const int zero = 0;
    KH_CUDA(cudaMemcpyToSymbol(sm100::kh_tc_error, &zero, sizeof(int)));
  }
  return v;
}

}  // namespace kh
