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
// Work: one CTA per (packed tile of 128 consecutive packed rows, group of HG heads). Short
// sequences share a tile; a pair of rows from different sequences is masked. The keys of a tile
// are the packed rows of every sequence its rows belong to (clamped to +-WINDOW around the tile
// on windowed layers), in tiles of 64; which of them are present and unmasked is computed once
// per CTA as bit masks. The work is (head, key tile) items on two streams: stream 0 takes the
// even heads of the CTA, stream 1 the odd ones, and their items alternate on the tensor core so
// each stream's softmax runs while the other's products do. With one head per CTA (small
// launches) the two streams split the head's key tiles and combine their partial results (split
// mode). 320 threads:
//   warp 0     TMA: Q of each head into its stream's slot, K and V of each item (64 rows) into
//              rings that run ahead across items;
//   warp 1     one thread issues S = Q K^T (M 128, N 64 keys, K = D) into the stream's TMEM
//              columns [64 g, 64 g + 64), two items ahead, and O += P V (M 128, N = D, K 64 keys,
//              V as an MN-major operand) into the stream's O columns [128 + D g, 128 + D g + D),
//              which accumulate over the key tiles of a head;
//   warps 2-9  softmax, warps 2-5 stream 0 and 6-9 stream 1, one thread per query row (TMEM
//              lane): the 64 scores in registers, the exponentials exp2(s - m) in the log2
//              domain against a reference point m that only moves when a tile's maximum exceeds
//              it by more than 8 (then O is rescaled in TMEM, which is rare), P in f16 into the
//              stream's shared-memory block (128-byte swizzled K-major rows); at the end of a
//              head, ctx = O / sum.
// Two CTAs share an SM (256 TMEM columns and <= 108 KB of shared memory each).

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "attn_tc.h"
#include "runtime.h"
#include "sm100.cuh"
#include "tmap.h"

namespace kh {

namespace {

using namespace sm100;

constexpr int TQ = 128;
constexpr int TK = 64;        // keys per item
constexpr int THREADS = 320;  // producer warp, MMA warp, two softmax warpgroups (one query row per thread)
constexpr uint32_t TMEM_COLS = 256;
constexpr int MAXKT = 320;  // key tiles of one CTA: sequences up to 20,480 rows

template <int D>
struct Cfg {
  static constexpr int ROW_BYTES = D * 2;     // one q / k / v row: the swizzle width
  static constexpr int QTILE = TQ * ROW_BYTES;  // 128 query rows
  static constexpr int KTILE = TK * ROW_BYTES;  // 64 key (or value) rows
  static constexpr int KS = D == 32 ? 4 : 2;  // K stages
  static constexpr int VS = D == 32 ? 4 : 2;  // V stages
  static constexpr int Q_OFF = 0;             // one Q tile per stream
  static constexpr int K_OFF = Q_OFF + 2 * QTILE;
  static constexpr int V_OFF = K_OFF + KS * KTILE;
  static constexpr int P_OFF = V_OFF + VS * KTILE;  // one P block per stream: 128 rows x 64 keys, 16 KB
  static constexpr int BITS_OFF = P_OFF + 2 * 16384;  // present-and-unmasked key bits [tile][2]
  // Row sums from the tensor core (P times a ones tile, 16 columns of TMEM per stream next to O)
  // instead of in the softmax threads: off. Each MMA instruction costs the issuing thread far
  // more than its tensor-core time at these sizes (measured: about 60 cycles per instruction for
  // M 128 x N 16..64 products), and the four sum MMAs per item measured 2.4 % slower overall
  // than the softmax threads' own additions.
  static constexpr bool SUMS = false;
  static constexpr int XCH_OFF = BITS_OFF + MAXKT * 2 * 4;  // split mode: m and l of both streams, f32 [2][2][128]
  static constexpr int LUT_OFF = XCH_OFF + 2 * 2 * 128 * 4;  // key masks of 4 bits as 4 words, [16]
  static constexpr int ONES_OFF = LUT_OFF + 16 * 16;
  static constexpr int BAR_OFF = ONES_OFF + (SUMS ? 2048 : 0);  // ones: 16 rows x 64 keys
  static constexpr int USED = BAR_OFF + 512;
  // at least 100 KB so that no more than two CTAs (2 x 256 TMEM columns) share an SM
  static constexpr int SMEM = (USED + 1024 > 102400 ? USED + 1024 : 102400);
  static constexpr uint64_t LAYOUT = D == 64 ? 2ull : 4ull;  // 128- or 64-byte swizzle
  static constexpr uint64_t SBO = (8 * ROW_BYTES) >> 4;       // 8-row group stride, 16-byte units
};

struct Params {
  const float* mask;
  const int32_t* seq_start;
  const int32_t* seq_len;
  const int32_t* row_seq;
  const int32_t* ptiles;
  __half* ctx;
  int H, HG, T, window;
  float scale_log2;  // SCALE * log2(e)
  // DeBERTa relative terms (REL kernels): per packed row [2][H][NP] f32 tables, c2p = q . posKey[p]
  // and p2c = k . posQuery[p], and the plan's relative index relidx [L][L] (local positions)
  const float* rel_tables;
  const uint32_t* relidx;
  const int32_t* rel1d;  // relidx as a function of i - j (null: use relidx)
  int L, NP;
};

template <int D>
__device__ __forceinline__ uint64_t desc_rows(const void* smem) {
  const uint64_t addr = smem_u32(smem);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (Cfg<D>::SBO << 32) | (1ull << 46) | (Cfg<D>::LAYOUT << 61);
}

template <int D, bool REL = false, bool SPLIT = false>
__global__ void __launch_bounds__(THREADS, 2) attn_tc_kernel(const __grid_constant__ CUtensorMap tmq,
                                                             const __grid_constant__ CUtensorMap tmkv, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sP = smem + C::P_OFF;
  uint32_t* vbits = reinterpret_cast<uint32_t*>(smem + C::BITS_OFF);  // [tile][2]: key present, unmasked
  // lut4[n]: the 4 keys of a nibble n of a keep mask as 32-bit masks (key kept: all ones)
  uint4* lut4 = reinterpret_cast<uint4*>(smem + C::LUT_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;             // [stream]
  uint64_t* q_empty = bars + 2;        // [stream]
  uint64_t* s_full = bars + 4;         // [stream]
  uint64_t* s_empty = bars + 6;        // [stream]
  uint64_t* p_full = bars + 8;         // [stream]
  uint64_t* o_full = bars + 10;        // [stream]
  uint64_t* drain = bars + 12;
  uint64_t* k_full = bars + 13;        // [KS]
  uint64_t* k_empty = k_full + C::KS;  // [KS]
  uint64_t* v_full = k_empty + C::KS;  // [VS]
  uint64_t* v_empty = v_full + C::VS;  // [VS]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(v_empty + C::VS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int H = p.H, HG = p.HG, hg0 = blockIdx.y * HG;
  const int q0 = p.ptiles[3 * tile];
  int kstart = p.ptiles[3 * tile + 1], kend = p.ptiles[3 * tile + 2];
  if (p.window > 0) {
    kstart = max(kstart, q0 - p.window);
    kend = min(kend, q0 + TQ + p.window);
  }
  const int nkt = min((kend - kstart + TK - 1) / TK, MAXKT);
  const int NI = HG * nkt;  // (head, key tile) items
  // The items in the order the producer and the MMA warp take them: heads in pairs (2a, 2a + 1),
  // the key tiles of the two alternating (stream 0 takes even heads, stream 1 odd ones); a last
  // head without a partner runs alone on stream 0. With one head per CTA (split mode: small
  // launches) the streams split the head's key tiles instead, stream g taking tiles j = g mod 2,
  // and combine their partial softmax results at the end.
  constexpr bool split = SPLIT;  // (launched with HG == 1)
  auto advance = [HG, nkt](int& hh, int& j, int& g) {
    if constexpr (split) {
      ++j;
      g ^= 1;
    } else if (g == 0 && hh + 1 < HG) {
      g = 1;
      ++hh;
    } else {
      if (g == 1) --hh;
      g = 0;
      if (++j == nkt) {
        j = 0;
        hh += 2;
      }
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_full[s], 1);
    }
    for (int s = 0; s < C::KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmkv);
  }
  if (threadIdx.x < 16) {
    const uint32_t n = threadIdx.x;
    lut4[n] = make_uint4((n & 1u) ? ~0u : 0u, (n & 2u) ? ~0u : 0u, (n & 4u) ? ~0u : 0u, (n & 8u) ? ~0u : 0u);
  }
  if constexpr (C::SUMS) {
    // B operand of the row-sum MMA: 16 x 64 f16 ones (every swizzle of it is the same)
    uint4* ones = reinterpret_cast<uint4*>(smem + C::ONES_OFF);
    for (int i = threadIdx.x; i < 2048 / 16; i += THREADS) ones[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      // issued loads not yet known complete: parity per ring slot (bit 2 = issued)
      uint32_t pend_q = 0, pend_k = 0, pend_v = 0;
      int qn0 = 0, qn1 = 0;  // heads loaded per stream
      int hh = 0, j = 0, g = 0;
      for (int it = 0; it < NI && ok; ++it, advance(hh, j, g)) {
        const int h = hg0 + hh;
        const int y = kstart + j * TK;
        if (split ? j < 2 : j == 0) {  // the stream's first item of the head: its Q tile
          const uint32_t u = uint32_t(g ? qn1++ : qn0++);
          if (*abort_flag || !mbar_wait(&q_empty[g], (u & 1) ^ 1, 20)) { ok = false; break; }
          mbar_arrive_expect_tx(&q_full[g], C::QTILE);
          tma_load_2d(sQ + g * C::QTILE, &tmq, &q_full[g], h * D, q0);
          pend_q = (pend_q & ~(7u << (3 * g))) | ((4u | (u & 1)) << (3 * g));
        }
        {
          const int s = it % C::KS;
          const uint32_t u = uint32_t(it / C::KS);
          if (*abort_flag || !mbar_wait(&k_empty[s], (u & 1) ^ 1, 21)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[s], C::KTILE);
          tma_load_2d(sK + s * C::KTILE, &tmkv, &k_full[s], (H + h) * D, y);
          pend_k = (pend_k & ~(7u << (3 * s))) | ((4u | (u & 1)) << (3 * s));
        }
        {
          const int s = it % C::VS;
          const uint32_t u = uint32_t(it / C::VS);
          if (*abort_flag || !mbar_wait(&v_empty[s], (u & 1) ^ 1, 22)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[s], C::KTILE);
          tma_load_2d(sV + s * C::KTILE, &tmkv, &v_full[s], (2 * H + h) * D, y);
          pend_v = (pend_v & ~(7u << (3 * s))) | ((4u | (u & 1)) << (3 * s));
        }
      }
      if (!ok) {
        *abort_flag = 1;
        // every copy this thread issued lands before the CTA ends
        for (int s = 0; s < 2; ++s)
          if ((pend_q >> (3 * s)) & 4u) mbar_wait(&q_full[s], (pend_q >> (3 * s)) & 1u, 31);
        for (int s = 0; s < C::KS; ++s)
          if ((pend_k >> (3 * s)) & 4u) mbar_wait(&k_full[s], (pend_k >> (3 * s)) & 1u, 32);
        for (int s = 0; s < C::VS; ++s)
          if ((pend_v >> (3 * s)) & 4u) mbar_wait(&v_full[s], (pend_v >> (3 * s)) & 1u, 33);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_f16(128, TK);
      const uint32_t idesc_o = idesc_f16(128, D) | (1u << 16);  // B (V) MN-major
      bool ok = true;
      int sh = 0, sj = 0, sg = 0;   // (head, key tile, stream) of the next S to issue
      int su0 = 0, su1 = 0, sq0 = 0, sq1 = 0;  // S issued / heads started per stream
      auto issue_s = [&](int it) -> bool {
        const int j = sj, g = sg;
        const int u = g ? su1++ : su0++;
        advance(sh, sj, sg);
        const int ks = it % C::KS;
        if (split ? j < 2 : j == 0) {
          const int qu = g ? sq1++ : sq0++;
          if (!mbar_wait(&q_full[g], uint32_t(qu) & 1, 23)) return false;
        }
        if (*abort_flag || !mbar_wait(&k_full[ks], uint32_t(it / C::KS) & 1, 24)) return false;
        if (*abort_flag || !mbar_wait(&s_empty[g], (uint32_t(u) & 1) ^ 1, 25)) return false;
        fence_after_sync();
        const uint64_t dq = desc_rows<D>(sQ + g * C::QTILE);
        const uint64_t dk = desc_rows<D>(sK + ks * C::KTILE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma_f16(tmem + uint32_t(g * TK), dq + uint64_t(2 * k), dk + uint64_t(2 * k), idesc_s, k ? 1u : 0u);
        mma_commit(&s_full[g]);
        mma_commit(&k_empty[ks]);
        if (split ? j + 2 >= nkt : j == nkt - 1) mma_commit(&q_empty[g]);  // the stream's last item of the head
        return true;
      };
      // S runs two items ahead of PV: the next item's S belongs to the other stream, the one
      // after to this stream, whose softmax can then start on it while its PV runs.
      ok = NI > 0 && issue_s(0);
      if (ok && NI > 1) ok = issue_s(1);
      int hh = 0, j = 0, g = 0;
      int pu0 = 0, pu1 = 0;
      for (int it = 0; it < NI && ok; ++it, advance(hh, j, g)) {
        if (it + 2 < NI && !issue_s(it + 2)) { ok = false; break; }
        const int u = g ? pu1++ : pu0++;
        const int vs = it % C::VS;
        if (*abort_flag || !mbar_wait(&p_full[g], uint32_t(u) & 1, 26) ||
            !mbar_wait(&v_full[vs], uint32_t(it / C::VS) & 1, 27)) {
          ok = false;
          break;
        }
        fence_after_sync();
        // O of the stream's head accumulates over its key tiles in the stream's TMEM buffer
        const uint32_t o_addr = tmem + 128 + uint32_t(g * D);
        const uint64_t dv = desc_rows<D>(sV + vs * C::KTILE);
        const uint64_t dp = desc_rows<64>(sP + g * 16384);
        const bool acc = split ? j >= 2 : j > 0;  // not the stream's first item of the head
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk)
          mma_f16(o_addr, dp + uint64_t(2 * kk), dv + uint64_t(2 * D * kk), idesc_o, (acc || kk) ? 1u : 0u);
        if constexpr (C::SUMS) {
          // row sums of P: P times the ones tile, accumulated like O
          const uint32_t l_addr = tmem + 192 + uint32_t(g * 16);
          const uint32_t idesc_l = idesc_f16(128, 16);
          const uint64_t d1 = desc_rows<64>(smem + C::ONES_OFF);
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk)
            mma_f16(l_addr, dp + uint64_t(2 * kk), d1 + uint64_t(2 * kk), idesc_l, (acc || kk) ? 1u : 0u);
        }
        mma_commit(&o_full[g]);
        mma_commit(&v_empty[vs]);
      }
      if (!ok) {
        *abort_flag = 1;
        mma_commit(drain);
        mbar_wait(drain, 0, 34);
      }
    }
  } else {
    // Softmax: warps 2-5 run stream 0 (even heads of the CTA), warps 6-9 stream 1 (odd heads),
    // one thread per query row (TMEM lane: warp % 4 gives the lane quarter) over the 64 keys of
    // every item. The two streams alternate on the tensor core and cover each other's waits.
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;     // query row = TMEM lane
    const int tid_g = ((warp - 2) & 3) * 32 + lane;  // 0 .. 127 within the stream
    const int tid = threadIdx.x - 64;            // 0 .. 255
    // which key rows of every key tile are present and unmasked (once for all heads)
    for (int j = tid >> 6; j < nkt; j += 4) {
      const int kk = kstart + j * TK + (tid & 63);
      const bool valid = kk < kend && kk < p.T && p.mask[kk] > 0.5f;
      const uint32_t vb = __ballot_sync(0xffffffffu, valid);
      if (lane == 0) vbits[j * 2 + ((tid & 63) >> 5)] = vb;
    }
    const int row = q0 + r_local;
    const bool in_range = row < p.T;
    const bool qvalid = in_range && p.mask[row] > 0.5f;
    // packed key rows this query may attend: its own sequence, clamped to the window
    int lo = 0, hi = 0, sstart = 0;
    if (qvalid) {
      const int s = p.row_seq[row];
      lo = p.seq_start[s];
      sstart = lo;
      hi = lo + p.seq_len[s];
      if (p.window > 0) {
        lo = max(lo, row - p.window);
        hi = min(hi, row + p.window + 1);
      }
    }
    named_bar(5, 256);
    const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t s_addr = trow + uint32_t(g * TK);
    const uint32_t o_addr = trow + 128 + uint32_t(g * D);
    const int vrow = tid_g & 63, vpart = tid_g >> 6;  // value row (and its half) this thread clears
    bool ok = true;
    auto wwait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      const bool r = !*abort_flag && mbar_wait(bar, parity, code);
      return __all_sync(0xffffffffu, r);
    };
    // PV products of this stream observed complete so far (o_full completes once per PV, in
    // order; the softmax observes PV(u - 1) before it releases item u, so the barrier is never
    // two phases ahead of the phase waited for)
    int o_done = 0;
    auto wait_pv = [&](int u) -> bool {
      while (o_done <= u) {
        if (!wwait(&o_full[g], uint32_t(o_done & 1), 43)) return false;
        ++o_done;
      }
      fence_after_sync();
      return true;
    };
    // context row of head hh = O / l (a masked query row, or one without a kept key, is exactly
    // zero: select, not multiply); with tensor-core sums l is read from TMEM
    auto finish_head = [&](int hh, float lt) {
      if constexpr (C::SUMS) {
        uint32_t lr[8];
        tmem_ld8(trow + 192 + uint32_t(g * 16), lr);
        tmem_ld_wait();
        lt = __uint_as_float(lr[0]);
      }
      const bool live = qvalid && lt > 0.f;
      const float inv = live ? 1.0f / lt : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.ctx + int64_t(row) * H * D + int64_t(hg0 + hh) * D);
#pragma unroll
      for (int c = 0; c < D; c += 8) {
        uint32_t r[8];
        tmem_ld8(o_addr + c, r);
        tmem_ld_wait();
        __half2 hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          hv[e] = live ? __floats2half2_rn(__uint_as_float(r[2 * e]) * inv, __uint_as_float(r[2 * e + 1]) * inv)
                       : __floats2half2_rn(0.f, 0.f);
        if (in_range) dst[c / 8] = *reinterpret_cast<uint4*>(hv);
      }
    };
    uint8_t* prow = sP + g * 16384 + r_local * 128;
    const int pairs = HG >> 1;  // full head pairs (their items alternate between the streams)
    int u = 0;                  // stream-local item index
    float l_prev = 0.f;
    // Running state of the current head: m = the reference point of the exponentials (scaled
    // log2 units), moved only when a key tile's maximum exceeds it by more than 8 (probabilities
    // stay <= 2^8, exact in f16 up to the rounding; O in TMEM is rescaled then); l = the row sum.
    bool started = false;
    float m = 0.f, l = 0.f;
    for (int hh = split ? 0 : g; hh < HG && ok; hh += 2) {
      started = false;
      m = 0.f;
      l = 0.f;
      const int base = (hh >> 1) * 2 * nkt;  // global index of the head pair's first item
      const bool paired = (hh >> 1) < pairs;
      for (int j = split ? g : 0; j < nkt; j += split ? 2 : 1, ++u) {
        // global item index
        const int it = split ? j : paired ? base + 2 * j + g : base + j;
        const int k0 = kstart + j * TK;
        const int clo = min(max(lo - k0, 0), 64), chi = min(max(hi - k0, 0), 64);
        // keep masks of the two 32-key chunks: in the row's key range, present, unmasked
        uint32_t km[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int a = min(max(clo - 32 * c, 0), 32), b = min(max(chi - 32 * c, 0), 32);
          const uint32_t below_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
          const uint32_t below_a = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
          km[c] = (below_b & ~below_a) & vbits[j * 2 + c];
        }
        if (!wwait(&s_full[g], uint32_t(u & 1), 41)) { ok = false; break; }
        uint32_t sr[64];
        fence_after_sync();
        tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(sr));
        tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tmem_ld_wait();
        fence_before_sync();
        mbar_arrive(&s_empty[g]);  // S in TMEM is free for this stream's next item
        if constexpr (REL) {
          // s = q.k + q.posKey[p] + k.posQuery[p], p = relidx[i][j] (local positions)
          if (p.rel1d) {
            // p depends on i - j only: p = rel1d[row - kj + L - 1]. Every key of a chunk with a kept
            // key gets the terms, four keys at a time with independent loads (for a fixed key the
            // warp's rows read neighbouring table entries); addresses are clamped to the rows and
            // the index range, and the scores of keys not kept are dropped to -inf below.
            const int rowc = min(row, p.T - 1);
            const float* c2p = p.rel_tables + (int64_t(rowc) * 2 * p.H + hg0 + hh) * p.NP;
            const float* p2c0 = p.rel_tables + (int64_t(p.H) + hg0 + hh) * p.NP;  // row 0's p2c of this head
            const int64_t rstride = int64_t(2) * p.H * p.NP;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              if (!__any_sync(0xffffffffu, km[c] != 0u)) continue;
#pragma unroll
              for (int g4 = 0; g4 < 32; g4 += 4) {
                int pp[4];
                int kc[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int kj = k0 + c * 32 + g4 + e;
                  kc[e] = min(kj, p.T - 1);
                  pp[e] = __ldg(p.rel1d + min(max(row - kj + p.L - 1, 0), 2 * p.L - 2));
                }
                float a[4], b[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  a[e] = __ldg(c2p + pp[e]);
                  b[e] = __ldg(p2c0 + int64_t(kc[e]) * rstride + pp[e]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int i = c * 32 + g4 + e;
                  sr[i] = __float_as_uint(__uint_as_float(sr[i]) + a[e] + b[e]);
                }
              }
            }
          } else {
          const float* c2p = p.rel_tables + (int64_t(row) * 2 * p.H + hg0 + hh) * p.NP;
          const uint32_t* ridx = p.relidx + int64_t(row - sstart) * p.L - sstart;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (!__any_sync(0xffffffffu, km[c] != 0u)) continue;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if ((km[c] >> i) & 1u) {
                const int kj = k0 + c * 32 + i;
                const uint32_t pp = __ldg(ridx + kj);
                const float* p2c = p.rel_tables + ((int64_t(kj) * 2 + 1) * p.H + hg0 + hh) * p.NP;
                sr[c * 32 + i] = __float_as_uint(__uint_as_float(sr[c * 32 + i]) + __ldg(c2p + pp) + __ldg(p2c + pp));
              }
            }
          }
          }
        }
        // warp-uniform cases per 32-key chunk: every lane keeps all keys, none keeps any, or mixed;
        // in a mixed chunk a dropped key's score becomes -inf ((s & mask) | (~mask & bits(-inf)),
        // whatever it was), so the maximum and the exponentials below need no masks
        bool any_c[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          any_c[c] = __any_sync(0xffffffffu, km[c] != 0u);
          if (any_c[c] && !__all_sync(0xffffffffu, km[c] == 0xffffffffu)) {
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const uint4 mk = lut4[(km[c] >> (4 * i4)) & 0xFu];
              const int i = 32 * c + 4 * i4;
              sr[i] = (sr[i] & mk.x) | (~mk.x & 0xFF800000u);
              sr[i + 1] = (sr[i + 1] & mk.y) | (~mk.y & 0xFF800000u);
              sr[i + 2] = (sr[i + 2] & mk.z) | (~mk.z & 0xFF800000u);
              sr[i + 3] = (sr[i + 3] & mk.w) | (~mk.w & 0xFF800000u);
            }
          }
        }
        // the row maximum of the kept raw scores
        float mr[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (any_c[c]) {
#pragma unroll
            for (int i = 0; i < 32; i += 2)
              mr[(i >> 1) & 3] = fmax3(mr[(i >> 1) & 3], __uint_as_float(sr[32 * c + i]), __uint_as_float(sr[32 * c + i + 1]));
          }
        }
        const float mraw = fmaxf(fmaxf(mr[0], mr[1]), fmaxf(mr[2], mr[3]));
        float corr = 1.f;
        if (mraw > -INFINITY) {
          const float cand = mraw * p.scale_log2;
          if (!started) {
            m = cand;
            started = true;
          } else if (cand > m + 8.f) {
            corr = ex2_approx(m - cand);
            m = cand;
          }
        }
        // P of this stream's previous item is free, and O holds all its products, once its PV
        // product is done (it has long been, as a rule)
        if (u >= 1 && !wait_pv(u - 1)) { ok = false; break; }
        if (!split && j == 0 && hh >= 2) finish_head(hh - 2, l_prev);  // before this head's first PV overwrites O
        if (__any_sync(0xffffffffu, corr != 1.f)) {
          // rescale O (the PV products so far) before this item's PV
#pragma unroll 1
          for (int c = 0; c < D; c += 8) {
            uint32_t r[8];
            tmem_ld8(o_addr + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
            tmem_st8(o_addr + c, r);
          }
          if constexpr (C::SUMS) {
            const uint32_t l_addr = trow + 192 + uint32_t(g * 16);
            uint32_t r[8];
            tmem_ld8(l_addr, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
            tmem_st8(l_addr, r);
          }
          tmem_st_wait();
        }
        // p = exp2(s scale log2e - m) in f16, into this row of the stream's P block (128-byte swizzled)
        float2 ls2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const bool any = any_c[c];
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // keys 8 q .. 8 q + 7 of the chunk: one 16-byte chunk of P
            uint32_t pk[4] = {0u, 0u, 0u, 0u};
            if (any) {  // (a dropped key's score is -inf: its exponential is 0)
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const int i = 8 * q + 2 * e2;
                const float2 xx = ffma2(make_float2(__uint_as_float(sr[32 * c + i]), __uint_as_float(sr[32 * c + i + 1])),
                                        make_float2(p.scale_log2, p.scale_log2), make_float2(-m, -m));
                const float x0 = ex2_approx(xx.x);
                const float x1 = ex2_approx(xx.y);
                if constexpr (!C::SUMS) {
                  ls2[(i >> 1) & 1] = fadd2(ls2[(i >> 1) & 1], make_float2(x0, x1));
                }
                __half2 hv = __floats2half2_rn(x0, x1);
                pk[e2] = *reinterpret_cast<uint32_t*>(&hv);
              }
            }
            const int ch = c * 4 + q;
            *reinterpret_cast<uint4*>(prow + ((ch ^ (r_local & 7)) * 16)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
        l = l * corr + ((ls2[0].x + ls2[0].y) + (ls2[1].x + ls2[1].y));  // (corr rescales the sum so far)
        // value rows of masked or absent keys become zero before the PV product (a tile whose 64
        // key rows are all present and unmasked, the rule in packed bulk runs, needs nothing:
        // the MMA thread itself waits for V)
        if ((vbits[j * 2] & vbits[j * 2 + 1]) != 0xffffffffu) {
          const int vs = it % C::VS;
          if (!wwait(&v_full[vs], uint32_t(it / C::VS) & 1, 42)) { ok = false; break; }
          if (!((vbits[j * 2 + (vrow >> 5)] >> (vrow & 31)) & 1u)) {
            uint4* vr = reinterpret_cast<uint4*>(sV + vs * C::KTILE + vrow * C::ROW_BYTES + vpart * (C::ROW_BYTES / 2));
#pragma unroll
            for (int q = 0; q < C::ROW_BYTES / 32; ++q) vr[q] = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
        fence_before_sync();
        mbar_arrive(&p_full[g]);
      }
      l_prev = l;
    }
    // the stream's last head, once its last PV product is done
    if (ok && u > 0) ok = wait_pv(u - 1);
    if constexpr (!split) {
      if (ok && u > 0) finish_head(g + 2 * ((HG - 1 - g) >> 1), l_prev);
    } else {
      // Combine the two streams' parts of the head: m = max(m0, m1), O = sum_g 2^(m_g - m) O_g,
      // l = sum_g 2^(m_g - m) l_g (a stream without a kept key, or without items, adds nothing:
      // select, not multiply, so its TMEM is never read into the sum). The thread of stream g
      // writes the columns [g D / 2, (g + 1) D / 2) of the row.
      float* xm = reinterpret_cast<float*>(smem + C::XCH_OFF);
      float* xl = xm + 2 * 128;
      xm[g * 128 + r_local] = (u > 0 && started) ? m : -INFINITY;
      if constexpr (!C::SUMS) xl[g * 128 + r_local] = l;
      if (named_bar_any(1 + quarter, 64, !ok)) {
        ok = false;
      } else {
        const float m0 = xm[r_local], m1 = xm[128 + r_local];
        const float mm = fmaxf(m0, m1);
        const bool use0 = m0 > -INFINITY, use1 = m1 > -INFINITY;
        const float f0 = use0 ? ex2_approx(m0 - mm) : 0.f, f1 = use1 ? ex2_approx(m1 - mm) : 0.f;
        float l0, l1;
        if constexpr (C::SUMS) {
          uint32_t r0[8], r1[8];
          tmem_ld8(trow + 192, r0);
          tmem_ld8(trow + 192 + 16, r1);
          tmem_ld_wait();
          l0 = __uint_as_float(r0[0]);
          l1 = __uint_as_float(r1[0]);
        } else {
          l0 = xl[r_local];
          l1 = xl[128 + r_local];
        }
        const float lt = (use0 ? f0 * l0 : 0.f) + (use1 ? f1 * l1 : 0.f);
        const bool live = qvalid && lt > 0.f;
        const float inv = live ? 1.0f / lt : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.ctx + int64_t(row) * H * D + int64_t(hg0) * D + g * (D / 2));
#pragma unroll
        for (int c = 0; c < D / 2; c += 8) {
          uint32_t a0[8], a1[8];
          tmem_ld8(trow + 128 + uint32_t(g * (D / 2) + c), a0);
          tmem_ld8(trow + 128 + uint32_t(D + g * (D / 2) + c), a1);
          tmem_ld_wait();
          __half2 hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float v[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const float o0 = use0 ? f0 * __uint_as_float(a0[2 * e + t]) : 0.f;
              const float o1 = use1 ? f1 * __uint_as_float(a1[2 * e + t]) : 0.f;
              v[t] = live ? (o0 + o1) * inv : 0.f;
            }
            hv[e] = __floats2half2_rn(v[0], v[1]);
          }
          if (in_range) dst[c / 8] = *reinterpret_cast<uint4*>(hv);
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    fence_after_sync();
    tmem_free(tmem, TMEM_COLS);
  }
}

// ---- DeBERTa relative-position tables on the tensor cores ----
//
// For every packed row r, head h and relative-position row p of the layer's posKey / posQuery
// [NP, H D] (f16): table[r][0][h][p] = q_r,h . posKey[p, h] (c2p) and table[r][1][h][p] =
// k_r,h . posQuery[p, h] (p2c), f32 (src/plan/layers.ts:61-80: the attrel PART 0 / 1 products).
// One CTA per (128 rows, 256 positions, table, head): one TMA load of each operand, M 128 x N 256
// x K 64 in four tcgen05 MMAs, the accumulator read back from TMEM and stored as f32 rows.
struct RelParams {
  float* out;
  int T, H, NP;
};

__global__ void __launch_bounds__(128) relpos_tables_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                                                            const __grid_constant__ CUtensorMap tm_pk,
                                                            const __grid_constant__ CUtensorMap tm_pq,
                                                            const RelParams rp) {
  constexpr int D = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;           // 128 rows x 64 f16, 128-byte swizzle
  uint8_t* sB = smem + 16384;   // 256 positions x 64 f16
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);
  uint64_t* full = bars;
  uint64_t* done = bars + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* bad = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * 128, p0 = blockIdx.y * 256;
  const int t = blockIdx.z / rp.H, h = blockIdx.z - t * rp.H;
  if (threadIdx.x == 0) {
    mbar_init(full, 1);
    mbar_init(done, 1);
    *bad = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_holder, 256);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(full, 16384 + 32768);
    tma_load_2d(sA, &tm_qkv, full, (t == 0 ? h : rp.H + h) * D, row0);
    tma_load_2d(sB, t == 0 ? &tm_pk : &tm_pq, full, h * D, p0);
    if (mbar_wait(full, 0, 71)) {
      fence_after_sync();
      const uint64_t da = desc_sw128(sA), db = desc_sw128(sB);
#pragma unroll
      for (int k = 0; k < D / 16; ++k) mma_f16(tmem, da + uint64_t(2 * k), db + uint64_t(2 * k), idesc_f16(128, 256), k ? 1u : 0u);
    } else {
      *bad = 1;  // the copies may still land: the commit below waits for nothing issued
    }
    mma_commit(done);
  }
  __syncwarp();
  const bool ok = mbar_wait(done, 0, 72) && !*bad;
  fence_after_sync();
  const int r = row0 + warp * 32 + lane;
  const uint32_t taddr = tmem + (uint32_t(warp * 32) << 16);
  float* dst = rp.out + ((int64_t(r) * 2 + t) * rp.H + h) * rp.NP + p0;
#pragma unroll 1
  for (int c = 0; c < 256; c += 32) {
    uint32_t v[32];
    tmem_ld32(taddr + c, v);
    tmem_ld_wait();
    if (ok && r < rp.T && p0 + c < rp.NP) {
      if (p0 + c + 32 <= rp.NP && (rp.NP & 3) == 0) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          reinterpret_cast<float4*>(dst + c)[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                                             __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (p0 + c + i < rp.NP) dst[c + i] = __uint_as_float(v[i]);
      }
    }
  }
  if (threadIdx.x == 0 && *bad) mbar_wait(full, 0, 73);  // the loads of a failed wait land before the exit
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_free(tmem, 256);
  }
}

// Heads per CTA: as many as keep every SM busy, up to 12 (the CTA computes the key masks of a
// tile once for all its heads, and fewer, longer CTAs measured faster), an even number so both
// softmax streams work; one head per CTA (split mode) for small launches.
int heads_per_cta(int H, int tiles) {
  const int sms = device_sms();  // of the current device
  for (int g = 12; g > 1; g -= 2)  // an even count keeps both softmax streams busy
    if (H % g == 0 && int64_t(tiles) * (H / g) >= int64_t(sms)) return g;
  return 1;  // one head per CTA: the two streams split its key tiles
}
template <int D, bool REL = false>
void launch_tc(const AttnArgs& a, const SeqTable& seq, int T, cudaStream_t st) {
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<D, REL, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM));
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<D, REL, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM));
    if (REL)
      KH_CUDA(cudaFuncSetAttribute(relpos_tables_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 49152 + 1024 + 64));
  });
  if constexpr (REL) {
    // c2p / p2c tables of every packed row and head first
    const uint64_t cols = uint64_t(3) * a.H * D, hd = uint64_t(a.H) * D;
    const CUtensorMap& tq = tensor_map_f16(a.qkv, uint64_t(T), cols, cols, D, 128, 128);
    const CUtensorMap& tk = tensor_map_f16(a.pos_key, uint64_t(a.np), hd, hd, D, 256, 128);
    const CUtensorMap& tp = tensor_map_f16(a.pos_query, uint64_t(a.np), hd, hd, D, 256, 128);
    RelParams rp;
    rp.out = a.rel_tables;
    rp.T = T;
    rp.H = a.H;
    rp.NP = a.np;
    const dim3 g((T + 127) / 128, (a.np + 255) / 256, 2 * a.H);
    relpos_tables_kernel<<<g, 128, 49152 + 1024 + 64, st>>>(tq, tk, tp, rp);
  }
  const uint64_t cols = uint64_t(3) * a.H * D;
  const CUtensorMap& tmq = tensor_map_f16(a.qkv, uint64_t(T), cols, cols, D, TQ, D * 2);
  const CUtensorMap& tmkv = tensor_map_f16(a.qkv, uint64_t(T), cols, cols, D, TK, D * 2);
  Params p;
  p.mask = a.mask;
  p.seq_start = seq.start;
  p.seq_len = seq.len;
  p.row_seq = seq.row_seq;
  p.ptiles = seq.ptiles;
  p.ctx = static_cast<__half*>(a.ctx);
  p.H = a.H;
  p.HG = heads_per_cta(a.H, seq.nptiles);
  p.T = T;
  p.window = a.window;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.rel_tables = a.rel_tables;
  p.relidx = a.relidx;
  p.rel1d = a.rel1d;
  p.L = a.L;
  p.NP = a.np;
  dim3 grid(seq.nptiles, a.H / p.HG);
  if (p.HG == 1) attn_tc_kernel<D, REL, true><<<grid, THREADS, Cfg<D>::SMEM, st>>>(tmq, tmkv, p);
  else attn_tc_kernel<D, REL, false><<<grid, THREADS, Cfg<D>::SMEM, st>>>(tmq, tmkv, p);
}

// ---- packed attention whose sequence table lives in static device memory ----
//
// kh_attention_f16_noalloc runs the kernel above on caller-owned device buffers and keeps the
// sequence table it needs in a file-scope device array, so the call allocates no device memory.
// Limits: NA_MAX_ROWS packed rows and NA_MAX_SEQS sequences per call.

constexpr int NA_MAX_ROWS = 65536;
constexpr int NA_MAX_SEQS = 4096;
constexpr int NA_LENS = 0;                                  // [NA_MAX_SEQS] lengths (from the host)
constexpr int NA_START = NA_LENS + NA_MAX_SEQS;             // [NA_MAX_SEQS] first packed row
constexpr int NA_ROWSEQ = NA_START + NA_MAX_SEQS;           // [NA_MAX_ROWS] sequence of each row
constexpr int NA_PTILES = NA_ROWSEQ + NA_MAX_ROWS;          // [NA_MAX_ROWS / 128][3] packed tiles
constexpr int NA_WORDS = NA_PTILES + 3 * (NA_MAX_ROWS / TQ);  // 140,800 words, 563,200 bytes

// Every word a call reads is written earlier in the same call (lengths by the host copy, the rest
// by the two setup kernels): nothing here has to start at zero.
static __device__ __align__(256) int32_t kh_attn_noalloc_scratch[NA_WORDS];

// One CTA of 1024 threads: exclusive prefix sum of the n <= 4096 lengths (sequence starts).
__global__ void noalloc_starts_kernel(int32_t* w, int n) {
  __shared__ int32_t part[1024];
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  int32_t sum = 0;
  for (int i = 0; i < per; ++i)
    if (b0 + i < n) sum += w[NA_LENS + b0 + i];
  part[threadIdx.x] = sum;
  __syncthreads();
  for (int off = 1; off < int(blockDim.x); off <<= 1) {
    const int32_t v = int(threadIdx.x) >= off ? part[threadIdx.x - off] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t run = part[threadIdx.x] - sum;
  for (int i = 0; i < per; ++i)
    if (b0 + i < n) {
      w[NA_START + b0 + i] = run;
      run += w[NA_LENS + b0 + i];
    }
}

// Thread per packed row: its sequence, and for the first row of each 128-row tile the tile's key
// range (its first row's sequence start to its last row's sequence end), as the plan path's
// sequence table holds them.
__global__ void noalloc_rows_kernel(int32_t* w, int n, int T) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= T) return;
  auto seq_of = [&](int row) {
    int lo = 0, hi = n - 1;  // lengths >= 1: starts strictly increase
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (w[NA_START + mid] <= row) lo = mid;
      else hi = mid - 1;
    }
    return lo;
  };
  const int s = seq_of(r);
  w[NA_ROWSEQ + r] = s;
  if (r % TQ == 0) {
    const int s1 = seq_of(min(T, r + TQ) - 1);
    int32_t* pt = w + NA_PTILES + 3 * (r / TQ);
    pt[0] = r;
    pt[1] = w[NA_START + s];
    pt[2] = w[NA_START + s1] + w[NA_LENS + s1];
  }
}

// Address of the scratch array on the current device; the first call on a device looks it up
// and sets the attention kernels' shared-memory limit.
int32_t* noalloc_scratch() {
  static std::mutex mu;
  static int32_t* per_device[64] = {};
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  if (!per_device[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, kh_attn_noalloc_scratch);
    if (e != cudaSuccess)
      throw CudaError(std::string("kh_attention_f16_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<32, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<32>::SMEM));
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<64, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<64>::SMEM));
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<32, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<32>::SMEM));
    KH_CUDA(cudaFuncSetAttribute(attn_tc_kernel<64, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<64>::SMEM));
    per_device[dev] = static_cast<int32_t*>(ptr);
  }
  return per_device[dev];
}

}  // namespace

void attention_f16_noalloc(const void* qkv, const float* mask, void* ctx, const int32_t* seq_lens, int n_seqs,
                           int H, int D, float scale, int window, cudaStream_t st) {
  if (!qkv || !mask || !ctx || !seq_lens) throw ArgError("kh_attention_f16_noalloc: null pointer argument");
  if (n_seqs < 1 || n_seqs > NA_MAX_SEQS)
    throw ArgError("kh_attention_f16_noalloc: n_seqs " + std::to_string(n_seqs) + " outside [1, " +
                   std::to_string(NA_MAX_SEQS) + "]");
  if (D != 32 && D != 64) throw ArgError("kh_attention_f16_noalloc: head_dim must be 32 or 64");
  if (H < 1) throw ArgError("kh_attention_f16_noalloc: heads must be >= 1");
  if (window < 0) throw ArgError("kh_attention_f16_noalloc: window must be >= 0");
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(ctx) & 15))
    throw ArgError("kh_attention_f16_noalloc: qkv and ctx must be 16-byte aligned");
  const int max_len = (MAXKT * TK - TQ) / 2;
  int64_t T = 0;
  for (int i = 0; i < n_seqs; ++i) {
    if (seq_lens[i] < 1 || seq_lens[i] > max_len)
      throw ArgError("kh_attention_f16_noalloc: sequence length " + std::to_string(seq_lens[i]) + " outside [1, " +
                     std::to_string(max_len) + "]");
    T += seq_lens[i];
  }
  if (T > NA_MAX_ROWS)
    throw ArgError("kh_attention_f16_noalloc: " + std::to_string(T) + " packed rows, at most " +
                   std::to_string(NA_MAX_ROWS));
  if (st) {
    // the scratch address and the tensor maps below belong to the current device
    int sdev = -1;
    KH_CUDA(cudaStreamGetDevice(st, &sdev));
    if (sdev != current_device())
      throw ArgError("kh_attention_f16_noalloc: the stream belongs to device " + std::to_string(sdev) +
                     ", the current device is " + std::to_string(current_device()));
  }
  int32_t* w = noalloc_scratch();
  KH_CUDA(cudaMemcpyAsync(w + NA_LENS, seq_lens, size_t(n_seqs) * 4, cudaMemcpyHostToDevice, st));
  noalloc_starts_kernel<<<1, 1024, 0, st>>>(w, n_seqs);
  noalloc_rows_kernel<<<int((T + 255) / 256), 256, 0, st>>>(w, n_seqs, int(T));
  CUtensorMap tmq, tmkv;
  const uint64_t cols = uint64_t(3) * H * D;
  encode_tensor_map_f16(&tmq, qkv, uint64_t(T), cols, cols, D, TQ, D * 2);
  encode_tensor_map_f16(&tmkv, qkv, uint64_t(T), cols, cols, D, TK, D * 2);
  Params p;
  p.mask = mask;
  p.seq_start = w + NA_START;
  p.seq_len = w + NA_LENS;
  p.row_seq = w + NA_ROWSEQ;
  p.ptiles = w + NA_PTILES;
  p.ctx = static_cast<__half*>(ctx);
  p.H = H;
  p.HG = heads_per_cta(H, int((T + TQ - 1) / TQ));
  p.T = int(T);
  p.window = window;
  p.scale_log2 = scale * 1.4426950408889634f;
  const dim3 grid(unsigned((T + TQ - 1) / TQ), unsigned(H / p.HG));
  const bool one = p.HG == 1;
  if (D == 64 && one) attn_tc_kernel<64, false, true><<<grid, THREADS, Cfg<64>::SMEM, st>>>(tmq, tmkv, p);
  else if (D == 64) attn_tc_kernel<64, false, false><<<grid, THREADS, Cfg<64>::SMEM, st>>>(tmq, tmkv, p);
  else if (one) attn_tc_kernel<32, false, true><<<grid, THREADS, Cfg<32>::SMEM, st>>>(tmq, tmkv, p);
  else attn_tc_kernel<32, false, false><<<grid, THREADS, Cfg<32>::SMEM, st>>>(tmq, tmkv, p);
  KH_CUDA(cudaGetLastError());
}

int attention_tile_q(bool) { return 64; }

bool attention_tc_supported(bool f16, const AttnArgs& a) {
  // the key rows of one packed tile must fit the CTA's key-tile masks; relative attention on the
  // tensor cores takes 64-wide heads (DeBERTa-v2/v3) and needs its tables (AttnArgs::rel_tables)
  if (!f16 || a.L > (MAXKT * TK - TQ) / 2) return false;
  if (a.rel) return a.D == 64 && a.np > 0;
  return a.D == 64 || a.D == 32;
}

int64_t attention_rel_table_floats_per_row(int H, int np) { return int64_t(2) * H * np; }

void launch_attention(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st) {
  if (seq.nptiles <= 0 && seq.ntiles <= 0) return;
  if (!attention_tc_supported(f16, a)) {
    launch_attention_simt(f16, a, seq, st);
    return;
  }
  if (seq.nptiles <= 0) return;
  const int T = a.rows;  // packed rows of the launch: the last packed tile ends at T
  if (a.rel) {
    if (!a.rel_tables) throw PlanError("relative attention on the tensor cores without its tables");
    launch_tc<64, true>(a, seq, T, st);
  } else if (a.D == 64) {
    launch_tc<64>(a, seq, T, st);
  } else {
    launch_tc<32>(a, seq, T, st);
  }
}

int attn_error_code() {
  // read and cleared (after a sync of the work that may have set it)
  int v = 0;
  KH_CUDA(cudaMemcpyFromSymbol(&v, sm100::kh_tc_error, sizeof(int)));
  if (v) {
    const int zero = 0;
    KH_CUDA(cudaMemcpyToSymbol(sm100::kh_tc_error, &zero, sizeof(int)));
  }
  return v;
}

namespace {
__global__ void wait_limit_selftest_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  // nothing arrives on the barrier: the wait runs out after limit_ns and records code 90
  if (threadIdx.x == 0) sm100::mbar_wait_for(&bar, 0, 90, limit_ns);
  __syncthreads();
}
}  // namespace

void launch_wait_limit_selftest(int limit_us, cudaStream_t st) {
  if (limit_us < 1 || limit_us > 1000000) throw ArgError("wait-limit self-test: limit_us outside [1, 1e6]");
  wait_limit_selftest_kernel<<<1, 32, 0, st>>>(1000ull * uint64_t(limit_us));
  KH_CUDA(cudaGetLastError());
}

int attention_status(cudaStream_t st) {
  KH_CUDA(cudaStreamSynchronize(st));
  return attn_error_code();
}

}  // namespace kh
