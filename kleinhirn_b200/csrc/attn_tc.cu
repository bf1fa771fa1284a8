// Attention of f16 plans on tcgen05 tensor cores (flash form), and the dispatch between it and the
// CUDA-core kernel (kernels.cu: f32 plans, DeBERTa's relative terms, head dimensions other than
// 32 and 64).
//
// Semantics (src/kernels/attsoftmax.wgsl, mbattention.wgsl, src/wasm/plan.ts:578-634,767-789):
// score = SCALE * q_i . k_j in f32; keys with mask 0, keys of another sequence and keys outside
// the sliding window (|i - j| > WINDOW, local positions) get probability exactly 0; a query row
// with mask 0 gets a zero context row; ctx = sum_j p_ij v_j with p the softmax over the kept
// keys. Masked value rows never enter a sum (they are zeroed before the PV product, as attpv.wgsl
// loads them as zero).
//
// Work: one CTA per (packed tile of 128 consecutive packed rows, head). Short sequences share a
// tile; a pair of rows from different sequences is masked. The keys of a tile are the packed rows
// of every sequence its rows belong to (clamped to +-WINDOW around the tile on windowed layers),
// in tiles of 128. 192 threads:
//   warp 0     TMA: the Q tile once, K tiles (2 stages), V tiles (1 stage) from the qkv rows;
//   warp 1     one thread issues S = Q K^T (M 128, N 128 keys, K = D) into TMEM columns
//              [0, 128) and O_j = P_j V_j (M 128, N = D, K 128 keys, V as an MN-major operand)
//              into TMEM columns [128, 128 + D);
//   warps 2-5  softmax, one thread per query row (TMEM lane): scores in the log2 domain, running
//              max and sum, P_j in f16 into shared memory (128-byte swizzled K-major rows), then
//              the context row accumulated in registers: o = o * exp2(m_old - m_new) + O_j.
// Two CTAs share an SM (256 TMEM columns and < 114 KB of shared memory each).

#include <algorithm>

#include "attn_tc.h"
#include "sm100.cuh"
#include "tmap.h"
#include "runtime.h"

namespace kh {

namespace {

using namespace sm100;

constexpr int TQ = 128;
constexpr int TKEYS = 128;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 256;

template <int D>
struct Cfg {
  static constexpr int ROW_BYTES = D * 2;          // one q / k / v row: the swizzle width
  static constexpr int TILE = 128 * ROW_BYTES;     // one 128-row tile
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = TILE;               // 2 stages
  static constexpr int V_OFF = 3 * TILE;
  static constexpr int P_OFF = 4 * TILE;           // 2 blocks of 128 rows x 64 keys, 16 KB each
  static constexpr int META_OFF = P_OFF + 32768;   // key sequence, mask, position: 3 x 128 words
  static constexpr int BAR_OFF = META_OFF + 3 * 512;
  static constexpr int USED = BAR_OFF + 256;
  // at least ~100 KB so that no more than two CTAs (2 x 256 TMEM columns) share an SM
  static constexpr int SMEM = (USED + 1024 > 102400 ? USED + 1024 : 102400);
  static constexpr uint64_t LAYOUT = D == 64 ? 2ull : 4ull;  // 128- or 64-byte swizzle
  static constexpr uint64_t SBO = (8 * ROW_BYTES) >> 4;       // 8-row group stride, 16-byte units
};

struct Params {
  const float* mask;
  const int32_t* seq_start;
  const int32_t* seq_len;
  const int32_t* row_seq;
  const int32_t* row_pos;
  const int32_t* ptiles;
  __half* ctx;
  int H, T, window;
  float scale_log2;  // SCALE * log2(e)
};

template <int D>
__device__ __forceinline__ uint64_t desc_rows(const void* smem) {
  const uint64_t addr = smem_u32(smem);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (Cfg<D>::SBO << 32) | (1ull << 46) | (Cfg<D>::LAYOUT << 61);
}

__device__ __forceinline__ void named_sync_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int D>
__global__ void __launch_bounds__(THREADS, 2) attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sP = smem + C::P_OFF;
  int* kvalid = reinterpret_cast<int*>(smem + C::META_OFF);  // key row present and unmasked
  volatile int* kholes = kvalid + 128;                         // per tile parity: a masked key exists
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // 2
  uint64_t* k_empty = bars + 3;  // 2
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 6;
  uint64_t* s_full = bars + 7;
  uint64_t* s_empty = bars + 8;
  uint64_t* p_full = bars + 9;
  uint64_t* o_full = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, h = blockIdx.y;
  const int H = p.H;
  const int q0 = p.ptiles[3 * tile];
  int kstart = p.ptiles[3 * tile + 1], kend = p.ptiles[3 * tile + 2];
  if (p.window > 0) {
    kstart = max(kstart, q0 - p.window);
    kend = min(kend, q0 + TQ + p.window);
  }
  const int nkt = (kend - kstart + TKEYS - 1) / TKEYS;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_empty, 128);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tm);
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      uint32_t pend_k = 0, pend_v = 0;  // last issued parity per K stage / the V stage, bit 2: issued
      mbar_arrive_expect_tx(q_full, C::TILE);
      tma_load_2d(sQ, &tm, q_full, h * D, q0);
      auto load_k = [&](int j) {
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1, 21)) return false;
        mbar_arrive_expect_tx(&k_full[s], C::TILE);
        tma_load_2d(sK + s * C::TILE, &tm, &k_full[s], (H + h) * D, kstart + j * TKEYS);
        pend_k = (pend_k & ~(3u << (2 * s))) | ((4u | uint32_t((j >> 1) & 1)) << (2 * s));
        return true;
      };
      ok = load_k(0);
      for (int j = 0; j < nkt && ok; ++j) {
        if (j + 1 < nkt && !load_k(j + 1)) ok = false;
        if (!ok || *abort_flag || !mbar_wait(v_empty, (j & 1) ^ 1, 22)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(v_full, C::TILE);
        tma_load_2d(sV, &tm, v_full, (2 * H + h) * D, kstart + j * TKEYS);
        pend_v = 4u | uint32_t(j & 1);
      }
      if (!ok) {
        *abort_flag = 1;
        mbar_wait(q_full, 0, 31);
        for (int s = 0; s < 2; ++s)
          if ((pend_k >> (2 * s)) & 4u) mbar_wait(&k_full[s], (pend_k >> (2 * s)) & 1u, 32);
        if (pend_v & 4u) mbar_wait(v_full, pend_v & 1u, 33);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_f16(128, TKEYS);
      const uint32_t idesc_o = idesc_f16(128, D) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, 23) && !*abort_flag;
      const uint64_t dq = desc_rows<D>(sQ);
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&k_full[s], (j >> 1) & 1, 24) || !mbar_wait(s_empty, (j & 1) ^ 1, 25)) {
          ok = false;
          break;
        }
        fence_after_sync();
        const uint64_t dk = desc_rows<D>(sK + s * C::TILE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) mma_f16(tmem, dq + uint64_t(2 * k), dk + uint64_t(2 * k), idesc_s, k ? 1u : 0u);
        mma_commit(s_full);
        mma_commit(&k_empty[s]);
        if (*abort_flag || !mbar_wait(p_full, j & 1, 26) || !mbar_wait(v_full, j & 1, 27)) {
          ok = false;
          break;
        }
        fence_after_sync();
        const uint64_t dv = desc_rows<D>(sV);
#pragma unroll
        for (int kk = 0; kk < TKEYS / 16; ++kk) {
          const uint64_t dp = desc_rows<64>(sP + (kk >> 2) * 16384) + uint64_t(2 * (kk & 3));
          mma_f16(tmem + 128, dp, dv + uint64_t(2 * D * kk), idesc_o, kk ? 1u : 0u);
        }
        mma_commit(o_full);
        mma_commit(v_empty);
      }
      if (!ok) {
        *abort_flag = 1;
        mma_commit(drain);
        mbar_wait(drain, 0, 34);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;  // query row = TMEM lane
    const int st = threadIdx.x - 64;          // key row this thread prepares
    const int row = q0 + r_local;
    const bool in_range = row < p.T;
    const bool qvalid = in_range && p.mask[row] > 0.5f;
    // packed key rows this query may attend: its own sequence, clamped to the window
    int lo = 0, hi = 0;
    if (qvalid) {
      const int s = p.row_seq[row];
      lo = p.seq_start[s];
      hi = lo + p.seq_len[s];
      if (p.window > 0) {
        lo = max(lo, row - p.window);
        hi = min(hi, row + p.window + 1);
      }
    }
    const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16);
    float m = -3.40282346638528859812e38f, l = 0.f;
    float o[D];
#pragma unroll
    for (int d = 0; d < D; ++d) o[d] = 0.f;
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      const int k0 = kstart + j * TKEYS;
      if (st == 0) kholes[j & 1] = 0;
      named_sync_softmax();
      {
        const int kk = k0 + st;
        const bool have = kk < kend && kk < p.T;
        const bool valid = have && p.mask[kk] > 0.5f;
        kvalid[st] = valid ? 1 : 0;
        if (have && !valid) kholes[j & 1] = 1;
      }
      named_sync_softmax();
      const bool holes = kholes[j & 1] != 0;
      const int clo = min(max(lo - k0, 0), TKEYS), chi = min(max(hi - k0, 0), TKEYS);
      if (*abort_flag || !mbar_wait(s_full, j & 1, 41)) {
        ok = false;
        break;
      }
      fence_after_sync();
      // pass 1: the row maximum of the kept raw scores
      float mraw = -3.40282346638528859812e38f;
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        const bool need = c4 * 32 < chi && c4 * 32 + 32 > clo;
        if (!__any_sync(0xffffffffu, need)) continue;
        uint32_t r[32];
        tmem_ld32(trow + c4 * 32, r);
        tmem_ld_wait();
        if (!need) continue;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = c4 * 32 + i;
          const bool keep = c >= clo && c < chi && (!holes || kvalid[c]);
          if (keep) mraw = fmaxf(mraw, __uint_as_float(r[i]));
        }
      }
      const float mx = fmaxf(m, mraw * p.scale_log2);
      const float corr = exp2f(m - mx);
      l *= corr;
      // pass 2: p = exp2(s scale log2e - max) in f16, into this row of P (128-byte swizzled)
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        const bool need = c4 * 32 < chi && c4 * 32 + 32 > clo;
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) packed[i] = 0u;
        if (__any_sync(0xffffffffu, need)) {
          uint32_t r[32];
          tmem_ld32(trow + c4 * 32, r);
          tmem_ld_wait();
          if (need) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float pv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int c = c4 * 32 + i + e;
                const bool keep = c >= clo && c < chi && (!holes || kvalid[c]);
                pv[e] = keep ? exp2f(fmaf(__uint_as_float(r[i + e]), p.scale_log2, -mx)) : 0.f;
                l += pv[e];
              }
              __half2 hv = __floats2half2_rn(pv[0], pv[1]);
              packed[i / 2] = *reinterpret_cast<uint32_t*>(&hv);
            }
          }
        }
        // keys c4*32 .. +31: block c4/2, 16-byte chunks 4 (c4 % 2) .. +3 of this row, swizzled
        uint8_t* prow = sP + (c4 >> 1) * 16384 + r_local * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (c4 & 1) * 4 + q;
          *reinterpret_cast<uint4*>(prow + ((ch ^ (r_local & 7)) * 16)) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      m = mx;
      fence_before_sync();
      mbar_arrive(s_empty);
      // value rows of masked or absent keys become zero before the PV product
      if (*abort_flag || !mbar_wait(v_full, j & 1, 42)) {
        ok = false;
        break;
      }
      if (!kvalid[st]) {
        uint4* vrow = reinterpret_cast<uint4*>(sV + st * C::ROW_BYTES);
#pragma unroll
        for (int q = 0; q < C::ROW_BYTES / 16; ++q) vrow[q] = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async();
      mbar_arrive(p_full);
      if (*abort_flag || !mbar_wait(o_full, j & 1, 43)) {
        ok = false;
        break;
      }
      fence_after_sync();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + 128 + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], corr, __uint_as_float(r[i]));
      }
    }
    if (!ok) *abort_flag = 1;
    if (in_range) {
      // a masked query row, or one without a kept key, is exactly zero (select, not multiply)
      const bool live = ok && qvalid && l > 0.f;
      const float inv = live ? 1.0f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.ctx + int64_t(row) * H * D + int64_t(h) * D);
#pragma unroll
      for (int q = 0; q < D / 8; ++q) {
        __half2 hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          hv[e] = live ? __floats2half2_rn(o[q * 8 + 2 * e] * inv, o[q * 8 + 2 * e + 1] * inv)
                       : __floats2half2_rn(0.f, 0.f);
        dst[q] = *reinterpret_cast<uint4*>(hv);
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    fence_after_sync();
    tmem_free(tmem, TMEM_COLS);
  }
}

template <int D>
void launch_tc(const AttnArgs& a, const SeqTable& seq, int T, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM));
    configured = true;
  }
  const uint64_t cols = uint64_t(3) * a.H * D;
  const CUtensorMap& tm = tensor_map_f16(a.qkv, uint64_t(T), cols, cols, D, 128, D * 2);
  Params p;
  p.mask = a.mask;
  p.seq_start = seq.start;
  p.seq_len = seq.len;
  p.row_seq = seq.row_seq;
  p.row_pos = seq.row_pos;
  p.ptiles = seq.ptiles;
  p.ctx = static_cast<__half*>(a.ctx);
  p.H = a.H;
  p.T = T;
  p.window = a.window;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  dim3 grid(seq.nptiles, a.H);
  attn_tc_kernel<D><<<grid, THREADS, Cfg<D>::SMEM, st>>>(tm, p);
}

}  // namespace

int attention_tile_q(bool) { return 64; }

bool attention_tc_supported(bool f16, const AttnArgs& a) { return f16 && !a.rel && (a.D == 64 || a.D == 32); }

void launch_attention(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st) {
  if (seq.nptiles <= 0) return;
  if (!attention_tc_supported(f16, a)) {
    launch_attention_simt(f16, a, seq, st);
    return;
  }
  // packed rows of the launch: the last packed tile ends at T
  const int T = a.rows;
  if (a.D == 64) launch_tc<64>(a, seq, T, st);
  else launch_tc<32>(a, seq, T, st);
}

int attn_error_code() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sm100::kh_tc_error, sizeof(int));
  return v;
}

}  // namespace kh
