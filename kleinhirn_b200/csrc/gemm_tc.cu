// tcgen05 GEMM of the encoder's projections: C = epilogue(A W^T + bias), A [M, K] f16 row-major
// (the activations), W [N, K] f16 row-major (PyTorch [out, in] weights, as the reference stores
// them, src/convert/names.ts:5), f32 accumulation in TMEM.
//
// Tiles are 256 x BN, computed by a cluster of two CTAs on two SMs (tcgen05 cta_group::2), with
// BN = 256 when N is a multiple of 256 or at least 1,024 (not GeGLU), else 192 when N is a
// multiple of 192, else 128. Each CTA
// stages its own 128 rows of A and BN / 2 rows of W; one thread of the first CTA issues the
// M = 256 MMAs, which read both CTAs' shared memory, and each CTA's TMEM holds its 128 rows of
// the accumulator. Per SM and K = 16 step the MMAs then read 4 KB of A and BN / 32 KB of W from
// shared memory (with one-SM 128 x BN tiles: 4 + BN / 16 KB), which together with the TMA writes
// stays within the SM's shared-memory bandwidth.
// Persistent: one cluster per SM pair, 64 + 128 BN / 64 threads per CTA in three roles:
//   warp 0      TMA producer (both CTAs): 128 x 64 tiles of A and BN / 2 x 64 tiles of W into a
//               ring of STAGES shared-memory stages (128-byte swizzle); both CTAs' bytes complete
//               on the first CTA's stage barrier;
//   warp 1      MMA issuer (first CTA): tcgen05.mma kind::f16 (M 256, N BN, K 16) into one of two
//               TMEM accumulators; each stage is committed back to both CTAs' producers and each
//               finished tile to both CTAs' epilogues;
//   warps 2..   epilogue, one warpgroup per 64 accumulator columns (warp w reads TMEM lanes
//               32 (w % 4) ..): bias, activation and the fused follow-up op in registers, the f16
//               result into a swizzled shared-memory tile, written out by one TMA store per
//               warpgroup (rows and columns past M and N are clipped by the tensor map).
// Tiles run n-fastest so the pairs working at the same time share rows of A in L2.
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
#include <atomic>
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

// Epilogue modes (compile time): 0-4 plain with activation ACT, then the fused follow-up ops.
enum EpiMode { EPI_MODE_RESIDUAL = 5, EPI_MODE_GEGLU = 6, EPI_MODE_ROPE = 7 };

struct Params {
  int M, N, K;
  const __half* bias;
  const float* table;
  const int32_t* row_pos;
  int rope_cols;  // columns of q and k (2 H D), heads of 64
};

// GELU with the Abramowitz-Stegun 7.1.26 erf (the reference's formula and constants,
// src/kernels/mmtile.wgsl:22-31): with u = v / sqrt(2), t = 1 / (1 + 0.3275911 |u|),
// p(t) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) and erf|u| = 1 - p(t) exp(-u^2), the reference's
// 0.5 v (1 + sign(v) erf|u|) equals relu(v) - 0.5 |v| p(t) exp(-v^2 / 2) for either sign of v,
// which takes fewer operations: the 1/sqrt(2) goes into the t constant, the 0.5 into the
// polynomial's coefficients. The reciprocal and exp use the MUFU approximations, whose error is
// far below the f16 rounding of the stored result.
__device__ __forceinline__ float gelu_as(float v) {
  const float a = fabsf(v);
  const float t = rcp_approx(fmaf(a, 0.3275911f * 0.7071067811865476f, 1.0f));
  float h = fmaf(0.5f * 1.061405429f, t, 0.5f * -1.453152027f);
  h = fmaf(h, t, 0.5f * 1.421413741f);
  h = fmaf(h, t, 0.5f * -0.284496736f);
  h = fmaf(h, t, 0.5f * 0.254829592f);
  const float hp = h * t;                                           // 0.5 p(t)
  const float e = ex2_approx((v * v) * (-0.5f * 1.4426950408889634f));  // exp(-v^2 / 2)
  return fmaf(-(a * hp), e, fmaxf(v, 0.0f));
}

// gelu_as on two values with packed f32x2 arithmetic (the same operations and roundings: the
// polynomial's coefficients carry the factor -0.5, so the last step is relu(v) + |v| (-hp) e).
__device__ __forceinline__ float2 gelu_as2(float2 v) {
  const float2 a = make_float2(fabsf(v.x), fabsf(v.y));
  const float2 d = ffma2(a, make_float2(0.3275911f * 0.7071067811865476f, 0.3275911f * 0.7071067811865476f),
                         make_float2(1.0f, 1.0f));
  const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  float2 h = ffma2(make_float2(-0.5f * 1.061405429f, -0.5f * 1.061405429f), t,
                   make_float2(-0.5f * -1.453152027f, -0.5f * -1.453152027f));
  h = ffma2(h, t, make_float2(-0.5f * 1.421413741f, -0.5f * 1.421413741f));
  h = ffma2(h, t, make_float2(-0.5f * -0.284496736f, -0.5f * -0.284496736f));
  h = ffma2(h, t, make_float2(-0.5f * 0.254829592f, -0.5f * 0.254829592f));
  const float2 nhp = fmul2(h, t);  // -0.5 p(t)
  const float2 w = fmul2(fmul2(v, v), make_float2(-0.5f * 1.4426950408889634f, -0.5f * 1.4426950408889634f));
  const float2 e = make_float2(ex2_approx(w.x), ex2_approx(w.y));
  return ffma2(fmul2(a, nhp), e, make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f)));
}

__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == 1) return fmaxf(v, 0.0f);
  if (act == 2) return gelu_as(v);
  if (act == 3) return tanhf(v);  // near 0 the exp form loses the relative precision f16 keeps
  if (act == 4) return v * rcp_approx(1.0f + ex2_approx(-v * 1.4426950408889634f));
  return v;
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

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

// Bias and activation of 32 accumulator columns [n, n + 32) of one row, in place.
template <int MODE>
__device__ __forceinline__ void bias_act32(float (&v)[32], const __half* bias, int n) {
  if (bias) {
    const uint4* s = reinterpret_cast<const uint4*>(bias + n);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = __ldg(s + q);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = fadd2(make_float2(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]), __half22float2(h[e]));
        v[q * 8 + 2 * e] = f.x;
        v[q * 8 + 2 * e + 1] = f.y;
      }
    }
  }
  if constexpr (MODE == 2) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float2 g = gelu_as2(make_float2(v[i], v[i + 1]));
      v[i] = g.x;
      v[i + 1] = g.y;
    }
  } else if constexpr (MODE >= 1 && MODE <= 4) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = act_fn(v[i], MODE);
  }
}

// ---- CTA pairs: 256 x BN tiles on two SMs (cta_group::2) ----
//
// A cluster of two CTAs computes a 256 x BN tile with one MMA stream: each CTA stages its own
// 128 rows of A and its own BN/2 rows of W, one thread of the first CTA issues M = 256 MMAs
// that read both CTAs' shared memory, and each CTA's TMEM receives its 128 rows of the
// accumulator. Per SM, one K = 16 step reads 4 KB of A and BN/32 KB of W from shared memory
// instead of 4 + BN/16 KB, which keeps the operand traffic of the MMAs and the TMA writes within
// the SM's shared-memory bandwidth.
template <int BN>
struct PCfg {
  static constexpr int BH = BN / 2;  // W rows staged per CTA
  static constexpr int B_BYTES = BH * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NWG = BN / 64;
  static constexpr int THREADS = 64 + 128 * NWG;
  static constexpr int SBUF = BN == 128 ? 2 : 1;
  static constexpr int STAGES = BN == 256 ? 5 : 6;  // as deep as the 227 KB of shared memory allow
  static constexpr uint32_t TMEM_COLS = BN == 128 ? 256 : 512;
  static constexpr int ACC_STRIDE = BN == 128 ? 128 : 256;  // TMEM columns between the two accumulators
  static constexpr int SMEM = STAGES * STAGE_BYTES + NWG * SBUF * OUT_BYTES + 1024 + 256;
};

template <int BN, int MODE>
__global__ void __launch_bounds__(PCfg<BN>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const Params p) {
  using G = PCfg<BN>;
  constexpr int STAGES = G::STAGES;
  constexpr int NWG = G::NWG;
  constexpr int SBUF = G::SBUF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * G::B_BYTES;  // [warpgroup][SBUF] 16 KB staging tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + NWG * SBUF * OUT_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* res_full = tempty + 2;
  uint64_t* drain = res_full + NWG;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool first = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (p.M + 2 * BM - 1) / (2 * BM), n_tiles = (p.N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * 4 * NWG);  // one arrival per epilogue warp of both CTAs
    }
    for (int g = 0; g < NWG; ++g) mbar_init(&res_full[g], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, G::TMEM_COLS);
  fence_before_sync();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int mb = t / n_tiles, nb = t % n_tiles;
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, 1)) {
            ok = false;
            break;
          }
          // both CTAs' bytes of the stage complete on the first CTA's barrier
          if (first) mbar_arrive_expect_tx(&full[stage], 2 * G::STAGE_BYTES);
          const uint32_t bar = cluster_addr(&full[stage], 0);
          tma_load_2d_pair(sA + stage * A_BYTES, &tmA, bar, kb * BK, mb * 2 * BM + int(rank) * BM);
          tma_load_2d_pair(sB + stage * G::B_BYTES, &tmB, bar, kb * BK, nb * BN + int(rank) * G::BH);
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
        // the first CTA's barriers count both CTAs' copies: wait for the ones issued
        if (first)
          for (int s = 0; s < STAGES; ++s)
            if (issued & (1u << s)) mbar_wait(&full[s], (last_parity >> s) & 1u, 11);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && first) {
      const uint32_t idesc = idesc_f16(2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++local) {
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[buf], tphase ^ 1, 2)) {
          ok = false;
          break;
        }
        fence_after_sync();
        const uint32_t d = tmem + uint32_t(buf * G::ACC_STRIDE);
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
            mma_f16_pair(d, da + uint64_t(k * 2), db + uint64_t(k * 2), idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit_pair_both(&empty[stage]);  // the stage is free again in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair_both(&tfull[buf]);
      }
      if (!ok) {
        *abort_flag = 1;
        mma_commit_pair(drain);  // the MMAs in flight finish before the TMEM is freed
        mbar_wait(drain, 0, 12);
      }
    }
  } else {
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const bool leader = (warp == 2 + 4 * g) && lane == 0;
    bool res_pending = false;
    uint32_t res_loads = 0;
    int local = 0;
    for (int t = pair; t < tiles; t += npairs, ++local) {
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      const int mb = t / n_tiles, nb = t % n_tiles;
      const int row0 = mb * 2 * BM + int(rank) * BM;  // first row of this CTA's half of the tile
      const int row = row0 + r;
      const bool live = row < p.M;
      const int n0 = nb * BN;
      uint8_t* stile = sOut + (g * SBUF + (local % SBUF)) * OUT_BYTES;
      const int nc = n0 + g * 64;
      if (leader) {
        bulk_wait_read<SBUF - 1>();
        if (MODE == EPI_MODE_RESIDUAL && nc < p.N) {
          mbar_arrive_expect_tx(&res_full[g], OUT_BYTES);
          tma_load_2d(stile, &tmC, &res_full[g], nc, row0);
          res_pending = true;
        }
      }
      const bool failed = *abort_flag || !mbar_wait(&tfull[buf], tphase, 4);
      if (named_bar_any(1 + g, 128, failed)) {
        *abort_flag = 1;
        break;
      }
      fence_after_sync();
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * G::ACC_STRIDE);
      // tells the MMA thread that this warp has read its accumulator rows
      auto release_acc = [&]() {
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[buf], 0));
      };
      if constexpr (MODE == EPI_MODE_GEGLU) {
        constexpr int OC = BN / 2 / NWG;  // outputs of one warpgroup: 32
        static_assert(OC == 32, "geglu warpgroups write 32 outputs");
        named_bar(1 + g, 128);  // the staging tile is free
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // 16 outputs at a time
          uint32_t ra[16], rb[16];
          tmem_ld16(taddr + g * 32 + 16 * half, ra);
          tmem_ld16(taddr + BN / 2 + g * 32 + 16 * half, rb);
          tmem_ld_wait();
          if (half == 1) release_acc();
          const uint4* ba = reinterpret_cast<const uint4*>(p.bias + n0 + g * 32 + 16 * half);
          const uint4* bb = reinterpret_cast<const uint4*>(p.bias + n0 + BN / 2 + g * 32 + 16 * half);
          uint32_t packed[8];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint4 ua = make_uint4(0, 0, 0, 0), ub = make_uint4(0, 0, 0, 0);
            if (p.bias) {
              ua = __ldg(ba + q);
              ub = __ldg(bb + q);
            }
            const __half2* ha = reinterpret_cast<const __half2*>(&ua);
            const __half2* hb = reinterpret_cast<const __half2*>(&ub);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = q * 8 + 2 * e;
              const float2 av = fadd2(make_float2(__uint_as_float(ra[i]), __uint_as_float(ra[i + 1])), __half22float2(ha[e]));
              const float2 bv = fadd2(make_float2(__uint_as_float(rb[i]), __uint_as_float(rb[i + 1])), __half22float2(hb[e]));
              const float2 gl = gelu_as2(make_float2(f16r(av.x), f16r(av.y)));
              const float2 o = fmul2(gl, make_float2(f16r(bv.x), f16r(bv.y)));
              __half2 h2 = __floats2half2_rn(o.x, o.y);
              packed[q * 4 + e] = *reinterpret_cast<uint32_t*>(&h2);
            }
          }
          // row r of the 64-byte-swizzled staging tile: 16-byte chunks 2 half, 2 half + 1
          uint8_t* row = stile + r * 64;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int ch = 2 * half + q;
            *reinterpret_cast<uint4*>(row + ((ch ^ ((r >> 1) & 3)) * 16)) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          }
        }
        fence_proxy_async_smem();
        named_bar(1 + g, 128);
        if (leader) {
          tma_store_2d(&tmC, stile, nb * (BN / 2) + g * 32, row0);
          bulk_commit();
        }
      } else if constexpr (MODE <= 4) {
        // bias + activation, 32 columns at a time (few registers live for the activation)
        const int nb0 = min(nc, p.N - 64);
        named_bar(1 + g, 128);  // the staging tile is free
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t ra[32];
          tmem_ld32(taddr + g * 64 + 32 * half, ra);
          tmem_ld_wait();
          if (half == 1) release_acc();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(ra[i]);
          bias_act32<MODE>(v, p.bias, nb0 + 32 * half);
          stage32_sw128(stile, r, 4 * half, v);
        }
        fence_proxy_async_smem();
        named_bar(1 + g, 128);
        if (leader) {
          if (nc < p.N) tma_store_2d(&tmC, stile, nc, row0);
          bulk_commit();
        }
      } else {
        uint32_t r0[32], r1[32];
        tmem_ld32(taddr + g * 64, r0);
        tmem_ld32(taddr + g * 64 + 32, r1);
        tmem_ld_wait();
        release_acc();
        float v0[32], v1[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v0[i] = __uint_as_float(r0[i]);
          v1[i] = __uint_as_float(r1[i]);
        }
        const int nb0 = min(nc, p.N - 64);
        if constexpr (MODE == EPI_MODE_ROPE) {
          bias_act32<0>(v0, p.bias, nb0);
          bias_act32<0>(v1, p.bias, nb0 + 32);
          if (nc < p.rope_cols) {
            const float4* tb = reinterpret_cast<const float4*>(p.table + int64_t(live ? p.row_pos[row] : 0) * 128);
#pragma unroll
            for (int d4 = 0; d4 < 8; ++d4) {
              const float4 c4 = __ldg(tb + d4), s4 = __ldg(tb + 16 + d4);
              const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int d = d4 * 4 + e;
                const float x = f16r(v0[d]), y = f16r(v1[d]);
                v0[d] = x * cs[e] - y * sn[e];
                v1[d] = y * cs[e] + x * sn[e];
              }
            }
          }
          named_bar(1 + g, 128);
        } else if constexpr (MODE == EPI_MODE_RESIDUAL) {
          bias_act32<0>(v0, p.bias, nb0);
          bias_act32<0>(v1, p.bias, nb0 + 32);
          if (nc < p.N) {
            if (!mbar_wait(&res_full[g], res_loads & 1u, 5)) *abort_flag = 1;
            ++res_loads;
            res_pending = false;
          }
          const uint8_t* srow = stile + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 u = *reinterpret_cast<const uint4*>(srow + ((c ^ (r & 7)) * 16));
            const __half2* h = reinterpret_cast<const __half2*>(&u);
            float* v = c < 4 ? v0 : v1;
            const int o = (c & 3) * 8;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(h[e]);
              v[o + 2 * e] = f.x + f16r(v[o + 2 * e]);
              v[o + 2 * e + 1] = f.y + f16r(v[o + 2 * e + 1]);
            }
          }
        }
        stage32_sw128(stile, r, 0, v0);
        stage32_sw128(stile, r, 4, v1);
        fence_proxy_async_smem();
        named_bar(1 + g, 128);
        if (leader) {
          if (nc < p.N) tma_store_2d(&tmC, stile, nc, row0);
          bulk_commit();
        }
      }
    }
    if (leader) {
      if (res_pending) mbar_wait(&res_full[g], res_loads & 1u, 13);
      bulk_wait<0>();
    }
  }
  fence_before_sync();
  cluster_sync();  // neither CTA leaves while the other may still use its shared memory or TMEM
  if (warp == 1) {
    fence_after_sync();
    tmem_free_pair(tmem, G::TMEM_COLS);
  }
}

// ---- GEMM + residual + LayerNorm (post-norm layers), on CTA pairs ----
//
// out = LayerNorm(R + round(A W^T + bias)) * w + b over rows of N = NF in {256, 384}: the matmul
// whose output only feeds a mode-2 layernorm (src/plan/layers.ts:118-149, attnOut + lnA and
// ffnOut + lnF) in one kernel. A pair owns whole 256-row tiles (all NF columns): two MMAs per
// K = 16 step, N = NF / 2 each, accumulate into TMEM columns [0, NF/2) and [256, 256 + NF/2); each
// CTA stages its 128 rows of the residual R by TMA into shared memory, and 16 epilogue warps
// (four column quarters per TMEM lane quarter) take three passes over their rows: (1) y =
// f16(acc + bias) from the accumulator into registers (packed halves, 48 per thread at NF 384)
// and the row sum of v = y + R; (2) the sum of squared deviations (the reference's two-pass
// variance, src/kernels/layernorm.wgsl:18-20); (3) the normalized f16 row, written over the
// staged R and stored by TMA. Passes 2 and 3 recompute v from y and R (exact: the same f32 sum),
// so the one accumulator is released after pass 1 and the next tile's MMAs run under them.
template <int NF>
struct LCfg {
  static constexpr int NH = NF / 2;                 // N of each of the two MMAs
  static constexpr int BQ = NF / 4;                 // W rows of one MMA staged per CTA
  static constexpr int B_BYTES = 2 * BQ * BK * 2;   // both boxes
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NBOX = NF / 64;              // 64-column boxes of a row tile
  static constexpr int X_BYTES = NBOX * OUT_BYTES;  // 128 rows x NF f16: residual in, result out
  static constexpr int STAGES = NF == 256 ? 4 : 3;
  static constexpr int THREADS = 64 + 512;
  static constexpr int RED_BYTES = 2 * 4 * 128 * 4;  // partial row sums [pass][quarter][row]
  static constexpr int VEC_BYTES = 3 * NF * 4;        // bias, ln_w, ln_b as f32
  static constexpr int SMEM = STAGES * STAGE_BYTES + X_BYTES + RED_BYTES + VEC_BYTES + 1024 + 256;
  static constexpr int D1 = 256;                    // TMEM column of the second MMA's accumulator
};

struct LnParams {
  int M, K;
  const __half* bias;  // matmul bias (or null)
  const __half* ln_w;
  const __half* ln_b;  // (or null)
  float eps;
};

template <int NF>
__global__ void __launch_bounds__(LCfg<NF>::THREADS, 1)
    gemm_addln_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmO,
                      const LnParams p) {
  using G = LCfg<NF>;
  constexpr int STAGES = G::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sX = sB + STAGES * G::B_BYTES;  // [box][128 rows][128 bytes], 128-byte swizzle
  float* red = reinterpret_cast<float*>(sX + G::X_BYTES);
  float* vbias = red + G::RED_BYTES / 4;  // [NF] matmul bias, then [NF] ln_w, [NF] ln_b, as f32
  float* vw = vbias + NF;
  float* vb = vw + NF;
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + G::RED_BYTES + G::VEC_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 1;
  uint64_t* res_full = tempty + 1;
  uint64_t* drain = res_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool first = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles = (p.M + 2 * BM - 1) / (2 * BM);
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 2 * 16);  // one arrival per epilogue warp of both CTAs
    mbar_init(res_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmR);
    prefetch_tmap(&tmO);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, 512);
  fence_before_sync();
  cluster_sync();
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, 51)) {
            ok = false;
            break;
          }
          if (first) mbar_arrive_expect_tx(&full[stage], 2 * G::STAGE_BYTES);
          const uint32_t bar = cluster_addr(&full[stage], 0);
          uint8_t* b = sB + stage * G::B_BYTES;
          tma_load_2d_pair(sA + stage * A_BYTES, &tmA, bar, kb * BK, t * 2 * BM + int(rank) * BM);
          tma_load_2d_pair(b, &tmB, bar, kb * BK, int(rank) * G::BQ);
          tma_load_2d_pair(b + G::BQ * 128, &tmB, bar, kb * BK, G::NH + int(rank) * G::BQ);
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
        if (first)
          for (int s = 0; s < STAGES; ++s)
            if (issued & (1u << s)) mbar_wait(&full[s], (last_parity >> s) & 1u, 61);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && first) {
      const uint32_t idesc = idesc_f16(2 * BM, G::NH);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++local) {
        if (*abort_flag || !mbar_wait(tempty, uint32_t(local & 1) ^ 1, 52)) {
          ok = false;
          break;
        }
        fence_after_sync();
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, 53)) {
            ok = false;
            break;
          }
          fence_after_sync();
          const uint64_t da = desc_sw128(sA + stage * A_BYTES);
          const uint64_t db0 = desc_sw128(sB + stage * G::B_BYTES);
          const uint64_t db1 = desc_sw128(sB + stage * G::B_BYTES + G::BQ * 128);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            mma_f16_pair(tmem, da + uint64_t(k * 2), db0 + uint64_t(k * 2), idesc, acc);
            mma_f16_pair(tmem + G::D1, da + uint64_t(k * 2), db1 + uint64_t(k * 2), idesc, acc);
          }
          mma_commit_pair_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair_both(tfull);
      }
      if (!ok) {
        *abort_flag = 1;
        mma_commit_pair(drain);
        mbar_wait(drain, 0, 62);
      }
    }
  } else {
    // warp w: TMEM lanes 32 (w % 4) .. (its rows), columns [g NF/4, (g + 1) NF/4)
    constexpr int QC = NF / 4;  // columns of one quarter: 64 or 96
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const bool leader = warp == 2 && lane == 0;
    const uint32_t trow = tmem + (uint32_t(q * 32) << 16);
    float* red1 = red;            // [quarter][row]: sums
    float* red2 = red + 4 * 128;  // [quarter][row]: squared deviations
    for (int i = threadIdx.x - 64; i < NF; i += 512) {  // seen by all after the first named barrier
      vbias[i] = p.bias ? __half2float(p.bias[i]) : 0.f;
      vw[i] = __half2float(p.ln_w[i]);
      vb[i] = p.ln_b ? __half2float(p.ln_b[i]) : 0.f;
    }
    bool res_pending = false;
    int local = 0;
    auto tcol = [&](int c0) { return trow + uint32_t(c0 < G::NH ? c0 : c0 - G::NH + G::D1); };
    constexpr int NP = QC / 16;   // 16-column pieces of a quarter: 4 or 6
    constexpr int NT = 4;         // pieces kept in TMEM
    constexpr int NR = NP - NT;   // pieces kept in registers: 0 or 2
    // y = f16(acc + bias) of this thread's row and quarter (packed halves, 8 words a piece) is
    // kept from pass 1 to pass 3: pieces 0-3 in the TMEM columns the accumulators leave free
    // (32 per quarter: [NF/2, 256) and [256 + NF/2, 512)), the rest in registers. The accumulator
    // is released after pass 1 and the next tile's MMAs run under the LayerNorm passes (v = y + R
    // is recomputed exactly from y and the staged R).
    const uint32_t ybase =
        trow + uint32_t(NF == 256 ? 128 + g * 32 : (g < 2 ? 192 + g * 32 : 448 + (g - 2) * 32));
    uint32_t yr[NR > 0 ? NR : 1][8];
    // v = y + R, f32, of the 16 columns of piece k (R from the staged residual)
    auto make_v = [&](int k, const uint32_t (&yk)[8], float (&v)[16]) {
      const int c0 = g * QC + k * 16;
      const uint8_t* xrow = sX + (c0 >> 6) * OUT_BYTES + r * 128;
      const int ch0 = (c0 & 63) >> 3;
#pragma unroll
      for (int cq = 0; cq < 2; ++cq) {
        const uint4 u = *reinterpret_cast<const uint4*>(xrow + (((ch0 + cq) ^ (r & 7)) * 16));
        const uint32_t rw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t yw = yk[cq * 4 + e];
          const float2 s = fadd2(__half22float2(*reinterpret_cast<const __half2*>(&yw)),
                                 __half22float2(*reinterpret_cast<const __half2*>(&rw[e])));
          v[cq * 8 + 2 * e] = s.x;
          v[cq * 8 + 2 * e + 1] = s.y;
        }
      }
    };
    // y of two pieces k0, k0 + 1 (one TMEM wait for both)
    auto load_y2 = [&](int k0, uint32_t (&y0)[8], uint32_t (&y1)[8]) {
      if (k0 < NT) {
        tmem_ld8(ybase + uint32_t(k0 * 8), y0);
        tmem_ld8(ybase + uint32_t(k0 * 8 + 8), y1);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          y0[i] = yr[k0 - NT][i];
          y1[i] = yr[k0 + 1 - NT][i];
        }
      }
    };
    for (int t = pair; t < tiles; t += npairs, ++local) {
      const int row0 = t * 2 * BM + int(rank) * BM;
      if (leader) {
        bulk_wait_read<0>();  // the previous tile's result has left the staging tile
        mbar_arrive_expect_tx(res_full, G::X_BYTES);
#pragma unroll
        for (int b = 0; b < G::NBOX; ++b) tma_load_2d(sX + b * OUT_BYTES, &tmR, res_full, b * 64, row0);
        res_pending = true;
        // short K: the residual of this CTA's next tile into L2 now, so that its load into the
        // staging tile (after this tile's result has left it) is an L2 hit; with long K the
        // loads of A keep HBM busy and the prefetch only competes with them
        if (p.K <= 512 && t + npairs < tiles) {
#pragma unroll
          for (int b = 0; b < G::NBOX; ++b) tma_prefetch_2d(&tmR, b * 64, row0 + npairs * 2 * BM);
        }
      }
      bool failed = *abort_flag || !mbar_wait(tfull, uint32_t(local & 1), 54);
      failed = failed || !mbar_wait(res_full, uint32_t(local & 1), 55);
      if (leader) res_pending = false;
      if (named_bar_any(1, 512, failed)) {
        *abort_flag = 1;
        break;
      }
      fence_after_sync();
      // pass 1: y from the accumulator, and this thread's statistics of v over its QC columns:
      // sums of d = v - c and d^2 around c = its first v (shifted sums, no cancellation to speak
      // of), merged over the four column quarters below (Chan, Golub and LeVeque's pairwise
      // update of means and squared deviations)
      float2 s2 = make_float2(0.f, 0.f), q2 = make_float2(0.f, 0.f);
      float c = 0.f;
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        const int c0 = g * QC + k * 16;
        uint32_t yk[8];
        {
          uint32_t a[16];
          tmem_ld16(tcol(c0), a);
          tmem_ld_wait();
          const float4* bs = reinterpret_cast<const float4*>(vbias + c0);
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const float4 b4 = bs[i4];
            const float2 p0 = fadd2(make_float2(__uint_as_float(a[4 * i4]), __uint_as_float(a[4 * i4 + 1])),
                                    make_float2(b4.x, b4.y));
            const float2 p1 = fadd2(make_float2(__uint_as_float(a[4 * i4 + 2]), __uint_as_float(a[4 * i4 + 3])),
                                    make_float2(b4.z, b4.w));
            const __half2 h0 = __floats2half2_rn(p0.x, p0.y), h1 = __floats2half2_rn(p1.x, p1.y);
            yk[2 * i4] = *reinterpret_cast<const uint32_t*>(&h0);
            yk[2 * i4 + 1] = *reinterpret_cast<const uint32_t*>(&h1);
          }
        }
        if (k < NT) {
          tmem_st8(ybase + uint32_t(k * 8), yk);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) yr[k - NT][i] = yk[i];
        }
        float v[16];
        make_v(k, yk, v);
        if (k == 0) c = v[0];
        const float2 nc = make_float2(-c, -c);
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float2 d = fadd2(make_float2(v[i], v[i + 1]), nc);
          s2 = fadd2(s2, d);
          q2 = ffma2(d, d, q2);
        }
      }
      // the accumulator is read (and y stored): the MMAs of the next tile may start
      tmem_st_wait();
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(tempty, 0));
      {
        const float s1 = s2.x + s2.y;
        red1[g * 128 + r] = c + s1 / float(QC);                            // mean of the quarter
        red2[g * 128 + r] = fmaxf((q2.x + q2.y) - s1 * (s1 / float(QC)), 0.f);  // its squared deviations
      }
      named_bar(1, 512);
      const float m0 = red1[r], m1 = red1[128 + r], m2 = red1[256 + r], m3 = red1[384 + r];
      const float mean = ((m0 + m1) + (m2 + m3)) * 0.25f;
      const float dm0 = m0 - mean, dm1 = m1 - mean, dm2 = m2 - mean, dm3 = m3 - mean;
      const float ssd = ((red2[r] + red2[128 + r]) + (red2[256 + r] + red2[384 + r])) +
                        float(QC) * ((dm0 * dm0 + dm1 * dm1) + (dm2 * dm2 + dm3 * dm3));
      const float var = ssd / float(NF);
      const float inv = 1.0f / sqrtf(var + p.eps);
      const float2 inv2 = make_float2(inv, inv), nmi2 = make_float2(-mean * inv, -mean * inv);
      // pass 3: (v - mean) inv w + b, written over the staged residual
      uint32_t y0[8], y1[8];
#pragma unroll
      for (int kk = 0; kk < NP; ++kk) {
        const int k = kk < NR ? NT + kk : kk - NR;  // the register pieces first (shorter live ranges)
        const int c0 = g * QC + k * 16;
        if ((k & 1) == 0) load_y2(k, y0, y1);
        float v[16];
        make_v(k, (k & 1) ? y1 : y0, v);
        uint8_t* xrow = sX + (c0 >> 6) * OUT_BYTES + r * 128;
        const int ch0 = (c0 & 63) >> 3;
#pragma unroll
        for (int cq = 0; cq < 2; ++cq) {
          const float4* w4 = reinterpret_cast<const float4*>(vw + c0 + cq * 8);
          const float4* b4 = reinterpret_cast<const float4*>(vb + c0 + cq * 8);
          const float4 wa = w4[0], wb = w4[1], ba = b4[0], bb = b4[1];
          const float2 wf[4] = {make_float2(wa.x, wa.y), make_float2(wa.z, wa.w), make_float2(wb.x, wb.y),
                                make_float2(wb.z, wb.w)};
          const float2 bf[4] = {make_float2(ba.x, ba.y), make_float2(ba.z, ba.w), make_float2(bb.x, bb.y),
                                make_float2(bb.z, bb.w)};
          __half2 o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // (v - mean) inv as v inv - mean inv: one rounding instead of two
            const float2 z = ffma2(ffma2(make_float2(v[cq * 8 + 2 * e], v[cq * 8 + 2 * e + 1]), inv2, nmi2), wf[e], bf[e]);
            o[e] = __floats2half2_rn(z.x, z.y);
          }
          *reinterpret_cast<uint4*>(xrow + (((ch0 + cq) ^ (r & 7)) * 16)) = *reinterpret_cast<uint4*>(o);
        }
      }
      fence_proxy_async_smem();
      named_bar(1, 512);
      if (leader) {
#pragma unroll
        for (int b = 0; b < G::NBOX; ++b) tma_store_2d(&tmO, sX + b * OUT_BYTES, b * 64, row0);
        bulk_commit();
      }
    }
    if (leader) {
      if (res_pending) mbar_wait(res_full, uint32_t(local & 1), 63);
      bulk_wait<0>();
    }
  }
  fence_before_sync();
  cluster_sync();
  if (warp == 1) {
    fence_after_sync();
    tmem_free_pair(tmem, 512);
  }
}

}  // namespace

bool gemm_tc_supported(int N, int K) { return N >= 64 && N % 64 == 0 && K % 8 == 0 && K >= 16; }
bool gemm_tc_supported_geglu(int N, int K) { return N % 128 == 0 && gemm_tc_supported(N, K); }
bool gemm_tc_supported_rope(int D) { return D == 64; }

// Tile width of a GEMM with N outputs (CTA-pair tiles: 256 x BN).
static int tile_n(int N) { return N % 256 == 0 ? 256 : (N % 192 == 0 ? 192 : 128); }

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

template <int BN, int MODE>
static void launch_pair_mode(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const Params& p,
                             int tiles, cudaStream_t st) {
  // resident CTA pairs per device (contexts of one process may drive several devices)
  static std::atomic<int> max_pairs_seen[64] = {};
  static std::atomic<uint64_t> configured{0};
  const int dev = current_device();
  once_per_device(configured, [dev] {
    KH_CUDA(cudaFuncSetAttribute(gemm_pair_kernel<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PCfg<BN>::SMEM));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * device_sms(), 1, 1);
    cfg.blockDim = dim3(PCfg<BN>::THREADS, 1, 1);
    cfg.dynamicSmemBytes = PCfg<BN>::SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    KH_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<BN, MODE>, &cfg));
    if (n <= 0) throw CudaError("gemm: no CTA pair fits on the device");
    max_pairs_seen[dev].store(n);
  });
  const int pairs = std::min(tiles, max_pairs_seen[dev].load());
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(PCfg<BN>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = PCfg<BN>::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  KH_CUDA(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<BN, MODE>, ma, mb, mc, p));
}

template <int BN>
static void launch_pair(const void* A, const void* W, void* C, const Params& p, int mode, cudaStream_t st) {
  const int M = p.M, N = p.N, K = p.K;
  const CUtensorMap& ma = tensor_map_f16(A, uint64_t(M), uint64_t(K), uint64_t(K), BK, BM, 128);
  const CUtensorMap& mb = tensor_map_f16(W, uint64_t(N), uint64_t(K), uint64_t(K), BK, BN / 2, 128);
  const CUtensorMap& mc = mode == EPI_MODE_GEGLU
                              ? tensor_map_f16(C, uint64_t(M), uint64_t(N / 2), uint64_t(N / 2), 32, 128, 64)
                              : tensor_map_f16(C, uint64_t(M), uint64_t(N), uint64_t(N), 64, 128, 128);
  const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
  switch (mode) {
    case 0: launch_pair_mode<BN, 0>(ma, mb, mc, p, tiles, st); break;
    case 1: launch_pair_mode<BN, 1>(ma, mb, mc, p, tiles, st); break;
    case 2: launch_pair_mode<BN, 2>(ma, mb, mc, p, tiles, st); break;
    case 3: launch_pair_mode<BN, 3>(ma, mb, mc, p, tiles, st); break;
    case 4: launch_pair_mode<BN, 4>(ma, mb, mc, p, tiles, st); break;
    case EPI_MODE_RESIDUAL: launch_pair_mode<BN, EPI_MODE_RESIDUAL>(ma, mb, mc, p, tiles, st); break;
    case EPI_MODE_GEGLU: launch_pair_mode<BN, EPI_MODE_GEGLU>(ma, mb, mc, p, tiles, st); break;
    case EPI_MODE_ROPE: launch_pair_mode<BN, EPI_MODE_ROPE>(ma, mb, mc, p, tiles, st); break;
    default: throw PlanError("gemm: unknown epilogue mode");
  }
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
  if (act < 0 || act > 4) throw PlanError("gemm: unknown activation " + std::to_string(act));
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.bias = static_cast<const __half*>(bias);
  p.table = nullptr;
  p.row_pos = nullptr;
  p.rope_cols = 0;
  int mode = act;
  if (e.kind == GemmEpilogue::Residual) {
    if (act) throw PlanError("residual epilogue after an activation");
    mode = EPI_MODE_RESIDUAL;
  } else if (e.kind == GemmEpilogue::GeGLU) {
    if (act) throw PlanError("geglu epilogue after an activation");
    mode = EPI_MODE_GEGLU;
  } else if (e.kind == GemmEpilogue::Rope) {
    if (e.D != 64) throw PlanError("rope epilogue needs 64-wide heads");
    if (act) throw PlanError("rope epilogue after an activation");
    mode = EPI_MODE_ROPE;
    p.table = e.table;
    p.row_pos = e.row_pos;
    p.rope_cols = 2 * e.H * e.D;
  }
  // Wide outputs take 256-column tiles even when N is not a multiple of 256 (the last tile's
  // warpgroups past N store nothing): for the qkv projection of N = 1,152 five such tiles per
  // row block ran 7 % faster than six 192-column ones. GeGLU keeps tile_n, which fixes the
  // weight's row interleave.
  const int bn = (mode != EPI_MODE_GEGLU && N >= 1024 && N % 256 != 0) ? 256 : tile_n(N);
  if (bn == 256) launch_pair<256>(A, W, C, p, mode, st);
  else if (bn == 192) launch_pair<192>(A, W, C, p, mode, st);
  else launch_pair<128>(A, W, C, p, mode, st);
}

bool gemm_tc_supported_addln(int N, int K) { return (N == 256 || N == 384) && K % 8 == 0 && K >= 16; }

template <int NF>
static void launch_addln_nf(const void* A, const void* W, const void* R, void* O, const LnParams& p,
                            cudaStream_t st) {
  using G = LCfg<NF>;
  // resident CTA pairs per device (contexts of one process may drive several devices)
  static std::atomic<int> max_pairs_seen[64] = {};
  static std::atomic<uint64_t> configured{0};
  const int dev = current_device();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  once_per_device(configured, [&attr, dev] {
    KH_CUDA(cudaFuncSetAttribute(gemm_addln_kernel<NF>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * device_sms(), 1, 1);
    cfg.blockDim = dim3(G::THREADS, 1, 1);
    cfg.dynamicSmemBytes = G::SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    KH_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_addln_kernel<NF>, &cfg));
    if (n <= 0) throw CudaError("gemm+layernorm: no CTA pair fits on the device");
    max_pairs_seen[dev].store(n);
  });
  const int max_pairs = max_pairs_seen[dev].load();
  const int M = p.M, K = p.K;
  const CUtensorMap& ma = tensor_map_f16(A, uint64_t(M), uint64_t(K), uint64_t(K), BK, BM, 128);
  const CUtensorMap& mb = tensor_map_f16(W, uint64_t(NF), uint64_t(K), uint64_t(K), BK, G::BQ, 128);
  const CUtensorMap& mr = tensor_map_f16(R, uint64_t(M), uint64_t(NF), uint64_t(NF), 64, 128, 128);
  const CUtensorMap& mo = tensor_map_f16(O, uint64_t(M), uint64_t(NF), uint64_t(NF), 64, 128, 128);
  const int tiles = (M + 2 * BM - 1) / (2 * BM);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * std::min(tiles, max_pairs), 1, 1);
  cfg.blockDim = dim3(G::THREADS, 1, 1);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  KH_CUDA(cudaLaunchKernelEx(&cfg, gemm_addln_kernel<NF>, ma, mb, mr, mo, p));
}

void launch_gemm_addln(const void* A, const void* W, const void* bias, const void* R, const void* ln_w,
                       const void* ln_b, float eps, void* O, int M, int N, int K, cudaStream_t st) {
  if (M <= 0) return;
  if (!gemm_tc_supported_addln(N, K)) throw PlanError("gemm+layernorm: unsupported shape");
  if (!ln_w) throw PlanError("gemm+layernorm: the norm weight is required");
  LnParams p;
  p.M = M;
  p.K = K;
  p.bias = static_cast<const __half*>(bias);
  p.ln_w = static_cast<const __half*>(ln_w);
  p.ln_b = static_cast<const __half*>(ln_b);
  p.eps = eps;
  if (N == 256) launch_addln_nf<256>(A, W, R, O, p, st);
  else launch_addln_nf<384>(A, W, R, O, p, st);
}

int tc_error_code() {
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
