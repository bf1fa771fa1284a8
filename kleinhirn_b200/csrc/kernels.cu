// Row kernels of the plan (bandwidth-bound) and the CUDA-core fallbacks of the contractions.
// Storage type T is __half for f16 plans and float for f32 plans; every kernel computes in f32
// and rounds once on store, as the reference kernels do (src/kernels/index.ts:1-3).
//
// Reference semantics per kernel are cited at each launcher. Row kernels use one warp per row
// with the row held in registers between the two LayerNorm passes (the variance is the mean of
// (v - mean)^2, src/kernels/layernorm.wgsl:18-20).

#include "act_f32.cuh"
#include "kernels.h"
#include "runtime.h"

#include <cmath>
#include <cstdio>
#include <stdexcept>

namespace kh {

namespace {

template <typename T> __device__ __forceinline__ float ld(const T* p, int64_t i);
template <> __device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <typename T> __device__ __forceinline__ void st(T* p, int64_t i, float v);
template <> __device__ __forceinline__ void st<float>(float* p, int64_t i, float v) { p[i] = v; }
template <> __device__ __forceinline__ void st<__half>(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

using f32act::activate;
using f32act::gelu_as;

constexpr int MAXE = 32;  // elements per lane held in registers: N <= 1024

// Two-pass LayerNorm over a row held as v[k] = x[lane + 32 k], k < n_per_lane.
__device__ __forceinline__ void ln_stats(const float* v, int N, float eps, float& mean, float& inv) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < MAXE; ++k) {
    const int d = lane + 32 * k;
    if (d < N) s += v[k];
  }
  mean = warp_sum(s) / float(N);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < MAXE; ++k) {
    const int d = lane + 32 * k;
    if (d < N) {
      const float x = v[k] - mean;
      q += x * x;
    }
  }
  const float var = warp_sum(q) / float(N);
  inv = 1.0f / sqrtf(var + eps);
}

template <typename T>
__global__ void embln_kernel(const T* __restrict__ word, const T* __restrict__ pos, const T* __restrict__ typ,
                             const uint32_t* __restrict__ tt, const T* __restrict__ w, const T* __restrict__ b,
                             const float* __restrict__ mask, T* __restrict__ out, int N, int rows,
                             const int32_t* __restrict__ row_pos, int offset, int maxpos, float eps, int maskmul,
                             int posids) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const uint32_t t = tt ? tt[row] : 0u;
  int prow = posids ? int(t >> 16) : row_pos[row] + offset;
  prow = min(prow, maxpos - 1);
  const int64_t wbase = int64_t(row) * N, pbase = int64_t(prow) * N, tbase = int64_t(t & 0xffffu) * N;
  float v[MAXE];
#pragma unroll
  for (int k = 0; k < MAXE; ++k) {
    const int d = lane + 32 * k;
    v[k] = d < N ? ld(word, wbase + d) + ld(pos, pbase + d) + ld(typ, tbase + d) : 0.f;
  }
  float mean, inv;
  ln_stats(v, N, eps, mean, inv);
  const float m = maskmul ? mask[row] : 1.0f;
#pragma unroll
  for (int k = 0; k < MAXE; ++k) {
    const int d = lane + 32 * k;
    if (d < N) {
      float y = (v[k] - mean) * inv * ld(w, d) + ld(b, d);
      if (maskmul) y *= m;
      st(out, wbase + d, y);
    }
  }
}

template <typename T>
__global__ void layernorm_kernel(const T* __restrict__ a, const T* __restrict__ bb, const T* __restrict__ w,
                                 const T* __restrict__ bias, const float* __restrict__ mask, T* __restrict__ out,
                                 int N, int rows, int mode, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t base = int64_t(row) * N;
  float v[MAXE];
#pragma unroll
  for (int k = 0; k < MAXE; ++k) {
    const int d = lane + 32 * k;
    float x = 0.f;
    if (d < N) {
      x = ld(a, base + d);
      if (mode == 2) x += ld(bb, base + d);
    }
    v[k] = x;
  }
  float mean, inv;
  ln_stats(v, N, eps, mean, inv);
  const float m = mode == 1 ? mask[row] : 1.0f;
#pragma unroll
  for (int k = 0; k < MAXE; ++k) {
    const int d = lane + 32 * k;
    if (d < N) {
      float y = (v[k] - mean) * inv * ld(w, d) + ld(bias, d);
      if (mode == 1) y *= m;
      st(out, base + d, y);
    }
  }
}

// Vectorised forms of the two row kernels: 16-byte loads and stores (8 f16 or 4 f32 per lane
// and step), one warp per row, the row in registers between the passes. N % (16 / sizeof(T)) == 0.
template <typename T> struct Vec;
template <> struct Vec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float* out) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      out[2 * e] = f.x;
      out[2 * e + 1] = f.y;
    }
  }
  __device__ static void store(__half* p, const float* v) {
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<uint4*>(h);
  }
};
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* out) {
    const float4 f = *reinterpret_cast<const float4*>(p);
    out[0] = f.x; out[1] = f.y; out[2] = f.z; out[3] = f.w;
  }
  __device__ static void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};

constexpr int MAXV = 4;  // vectors per lane: N <= 32 * 4 * 8 (f16) or 32 * 4 * 4 (f32)

// Groups of LPR lanes (8, 16 or 32) own one row each: lane i of a group holds vectors
// i, i + LPR, ... (v[k] = vector i + LPR k) and the reductions stay inside the group.
template <int LPR>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int LPR>
__device__ __forceinline__ void ln_vec_finish(float (&v)[MAXV][8], int N, const T* __restrict__ w,
                                              const T* __restrict__ bias, float eps, float scale, T* __restrict__ out,
                                              bool live) {
  constexpr int VN = Vec<T>::N;
  const int gl = threadIdx.x & (LPR - 1);
  const int nv = N / VN;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k)
    if (gl + LPR * k < nv)
#pragma unroll
      for (int e = 0; e < VN; ++e) s += v[k][e];
  const float mean = group_sum<LPR>(s) / float(N);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k)
    if (gl + LPR * k < nv)
#pragma unroll
      for (int e = 0; e < VN; ++e) {
        const float x = v[k][e] - mean;
        q += x * x;
      }
  const float inv = 1.0f / sqrtf(group_sum<LPR>(q) / float(N) + eps);
  if (!live) return;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int idx = gl + LPR * k;
    if (idx < nv) {
      float wv[8], bv[8], y[8];
      Vec<T>::load(w + idx * VN, wv);
      Vec<T>::load(bias + idx * VN, bv);
#pragma unroll
      for (int e = 0; e < VN; ++e) y[e] = ((v[k][e] - mean) * inv * wv[e] + bv[e]) * scale;
      Vec<T>::store(out + idx * VN, y);
    }
  }
}

template <typename T, int LPR>
__global__ void layernorm_vec_kernel(const T* __restrict__ a, const T* __restrict__ bb, const T* __restrict__ w,
                                     const T* __restrict__ bias, const float* __restrict__ mask, T* __restrict__ out,
                                     int N, int rows, int mode, float eps) {
  constexpr int VN = Vec<T>::N;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / LPR;
  const bool live = row < rows;  // every lane of a warp takes part in the shuffles
  const int gl = threadIdx.x & (LPR - 1);
  const int nv = N / VN;
  const int64_t base = int64_t(live ? row : 0) * N;
  float v[MAXV][8];
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int idx = gl + LPR * k;
    if (idx < nv) {
      Vec<T>::load(a + base + idx * VN, v[k]);
      if (mode == 2) {
        float y[8];
        Vec<T>::load(bb + base + idx * VN, y);
#pragma unroll
        for (int e = 0; e < VN; ++e) v[k][e] += y[e];
      }
    }
  }
  ln_vec_finish<T, LPR>(v, N, w, bias, eps, (mode == 1 && live) ? mask[row] : 1.0f, out + base, live);
}

template <typename T, int LPR>
__global__ void embln_vec_kernel(const T* __restrict__ word, const T* __restrict__ pos, const T* __restrict__ typ,
                                 const uint32_t* __restrict__ tt, const T* __restrict__ w, const T* __restrict__ b,
                                 const float* __restrict__ mask, T* __restrict__ out, int N, int rows,
                                 const int32_t* __restrict__ row_pos, int offset, int maxpos, float eps, int maskmul,
                                 int posids) {
  constexpr int VN = Vec<T>::N;
  const int row0 = (blockIdx.x * blockDim.x + threadIdx.x) / LPR;
  const bool live = row0 < rows;
  const int row = live ? row0 : 0;
  const int gl = threadIdx.x & (LPR - 1);
  const uint32_t t = tt ? tt[row] : 0u;
  int prow = posids ? int(t >> 16) : row_pos[row] + offset;
  prow = min(prow, maxpos - 1);
  const int64_t wbase = int64_t(row) * N, pbase = int64_t(prow) * N, tbase = int64_t(t & 0xffffu) * N;
  const int nv = N / VN;
  float v[MAXV][8];
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int idx = gl + LPR * k;
    if (idx < nv) {
      float x[8], y[8], z[8];
      Vec<T>::load(word + wbase + idx * VN, x);
      Vec<T>::load(pos + pbase + idx * VN, y);
      Vec<T>::load(typ + tbase + idx * VN, z);
#pragma unroll
      for (int e = 0; e < VN; ++e) v[k][e] = x[e] + y[e] + z[e];
    }
  }
  ln_vec_finish<T, LPR>(v, N, w, b, eps, (maskmul && live) ? mask[row] : 1.0f, out + wbase, live);
}

// Lanes per row of the vectorised row kernels: the fewest with at most MAXV vectors each.
inline int lanes_per_row(int nv) { return nv <= 8 * MAXV ? 8 : nv <= 16 * MAXV ? 16 : 32; }

template <typename T>
__global__ void add_kernel(T* __restrict__ dst, const T* __restrict__ src, int64_t count) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
    st(dst, i, ld(dst, i) + ld(src, i));
}

template <typename T>
__global__ void add_rows_kernel(T* __restrict__ dst, const T* __restrict__ src, int N, int rows,
                                const int32_t* __restrict__ row_seq) {
  const int64_t count = int64_t(rows) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / N;
    st(dst, i, ld(dst, i) + ld(src, int64_t(row_seq[r]) * N + (i - r * N)));
  }
}

template <typename T>
__global__ void geglu_kernel(const T* __restrict__ mid, T* __restrict__ gate, int I, int rows) {
  const int64_t total = int64_t(rows) * I;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / I;
    const int j = int(i - r * I);
    st(gate, i, gelu_as(ld(mid, r * 2 * I + j)) * ld(mid, r * 2 * I + I + j));
  }
}

template <typename T>
__global__ void rope_kernel(T* __restrict__ qkv, const float* __restrict__ cossin, const int32_t* __restrict__ row_pos,
                            int H, int D, int rows) {
  const int half = D / 2;
  const int64_t total = int64_t(rows) * 2 * H * half;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int d = int(idx % half);
    const int64_t rs = idx / half;
    const int s = int(rs % (2 * H));
    const int64_t i = rs / (2 * H);
    const int il = row_pos[i];
    const int64_t base = i * 3 * H * D + int64_t(s) * D;
    const float a = ld(qkv, base + d), b = ld(qkv, base + d + half);
    const float c = cossin[int64_t(il) * 2 * D + d], sn = cossin[int64_t(il) * 2 * D + D + d];
    st(qkv, base + d, a * c - b * sn);
    st(qkv, base + d + half, b * c + a * sn);
  }
}

template <typename T>
__global__ void pool_kernel(const T* __restrict__ x, const float* __restrict__ mask, T* __restrict__ out, int N,
                            int mode, const int32_t* __restrict__ start, const int32_t* __restrict__ len) {
  const int s = blockIdx.y;
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= N) return;
  const int r0 = start[s], n = len[s];
  if (mode == 0) {
    float acc = 0.f, cnt = 0.f;
    for (int i = 0; i < n; ++i) {
      const float m = mask[r0 + i];
      if (m != 0.f) {
        acc += m * ld(x, int64_t(r0 + i) * N + d);
        cnt += m;
      }
    }
    st(out, int64_t(s) * N + d, acc / fmaxf(cnt, 1e-9f));
  } else {
    float best = 0.f;
    bool found = false;
    for (int i = 0; i < n; ++i) {
      if (mask[r0 + i] > 0.5f) {
        const float v = ld(x, int64_t(r0 + i) * N + d);
        best = found ? fmaxf(best, v) : v;
        found = true;
      }
    }
    st(out, int64_t(s) * N + d, best);
  }
}

template <typename T>
__global__ void gather_kernel(const T* __restrict__ x, T* __restrict__ out, int D, const int32_t* __restrict__ start,
                              const int32_t* __restrict__ len, const uint32_t* __restrict__ markers, int K, int S) {
  const int g = blockIdx.x;  // output row
  const int s = g / K;
  if (s >= S) return;
  const uint32_t local = markers ? markers[s * 3 * K + (g - s * K)] : 0u;
  // a marker past the rows this call computed reads zeros (the reference reads whatever that
  // row of its buffer last held)
  const bool ok = local < uint32_t(len[s]);
  const int64_t row = int64_t(start[s]) + (ok ? local : 0);
  for (int d = threadIdx.x; d < D; d += blockDim.x) st(out, int64_t(g) * D + d, ok ? ld(x, row * D + d) : 0.f);
}

// logits[k] = raw[k] / temp where the marker's mask word (f32 bits) is above 0.5, else -1e4;
// the payload holds 3 K words per sequence: indices, mask, groups (src/kernels/masklogits.wgsl).
template <typename T>
__global__ void masklogits_kernel(const T* __restrict__ raw, const uint32_t* __restrict__ packed,
                                  float* __restrict__ logits, int K, float temp, int total) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= total) return;
  const int b = k / K;
  const float m = __uint_as_float(packed[b * 3 * K + K + (k - b * K)]);
  logits[k] = m > 0.5f ? ld(raw, k) / temp : -1e4f;
}

template <typename T>
__global__ void im2col_kernel(const T* __restrict__ x, const float* __restrict__ mask, T* __restrict__ out, int N,
                              int KS, int rows, const int32_t* __restrict__ start, const int32_t* __restrict__ len,
                              const int32_t* __restrict__ row_seq, const int32_t* __restrict__ row_pos) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int s = row_seq[r], i = row_pos[r], L = len[s], base = start[s];
  const int pad = (KS - 1) / 2;
  for (int t = 0; t < KS; ++t) {
    const int j = i + t - pad;
    const int src = base + max(j, 0);
    const bool ok = j >= 0 && j < L && mask[src] != 0.f;
    for (int c = threadIdx.x; c < N; c += blockDim.x)
      st(out, int64_t(r) * KS * N + int64_t(t) * N + c, ok ? ld(x, int64_t(src) * N + c) : 0.f);
  }
}

// C = act(A W^T + bias): TS x TS tiles (64, or 32 when 64-wide tiles would leave SMs idle), 256
// threads with (TS / 16) x (TS / 16) outputs each, k in steps of 16.
template <typename T, int TS>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ W,
                                                        const T* __restrict__ bias, T* __restrict__ C, int M, int N,
                                                        int K, int act) {
  constexpr int R = TS / 16;  // outputs per thread in each direction
  __shared__ float sa[16][TS + 1];
  __shared__ float sw[16][TS + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * TS, n0 = blockIdx.x * TS;
  float acc[R][R] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < TS * 16; e += 256) {
      const int r = e / 16, kk = e % 16;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      sa[kk][r] = (gm < M && gk < K) ? ld(A, int64_t(gm) * K + gk) : 0.f;
      sw[kk][r] = (gn < N && gk < K) ? ld(W, int64_t(gn) * K + gk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[R], b[R];
#pragma unroll
      for (int i = 0; i < R; ++i) a[i] = sa[kk][ty * R + i];
#pragma unroll
      for (int j = 0; j < R; ++j) b[j] = sw[kk][tx * R + j];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int gm = m0 + ty * R + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int gn = n0 + tx * R + j;
      if (gn < N) st(C, int64_t(gm) * N + gn, activate(acc[i][j] + (bias ? ld(bias, gn) : 0.f), act));
    }
  }
}

// Attention on CUDA cores, one warp per (query row, head): the lanes take the keys 32 at a time
// (lane l the key j0 + l: its score, with DeBERTa's relative terms), the chunk enters an online
// softmax in f32, and for the PV sum each lane owns the output dimensions l and l + 32. Keys with
// mask 0, outside the window or past the sequence are skipped (their value rows may hold NaN).
constexpr int AW = 16;          // warps (query rows) per CTA
constexpr int AROWS_TILE = 64;  // rows of one work tile of the sequence table (attention_tile_q)

template <typename T>
__global__ void __launch_bounds__(AW * 32) attention_simt_kernel(AttnArgs a, SeqTable seq) {
  const int tile = blockIdx.x / (AROWS_TILE / AW), sub = blockIdx.x % (AROWS_TILE / AW);
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = seq.tiles[2 * tile], q0 = seq.tiles[2 * tile + 1];
  const int base = seq.start[s], n = seq.len[s];
  const int H = a.H, D = a.D, hd = H * D;
  const T* qkv = static_cast<const T*>(a.qkv);
  T* ctx = static_cast<T*>(a.ctx);
  __shared__ float sq[AW][64];
  const int i = q0 + sub * AW + warp;  // local query
  if (i >= n) return;                  // (warp-uniform)
  const int64_t qrow = int64_t(base) + i;
  for (int d = lane; d < D; d += 32) sq[warp][d] = ld(qkv, qrow * 3 * hd + int64_t(h) * D + d);
  __syncwarp();
  const float* q = sq[warp];
  const bool qvalid = a.mask[qrow] > 0.5f;
  const T* pk = static_cast<const T*>(a.pos_key);
  const T* pq = static_cast<const T*>(a.pos_query);
  float m = -3.40282346638528859812e38f, l = 0.f, acc0 = 0.f, acc1 = 0.f;
  for (int j0 = 0; qvalid && j0 < n; j0 += 32) {
    const int j = j0 + lane;
    const bool keep = j < n && a.mask[base + j] > 0.5f && !(a.window && abs(i - j) > a.window);
    float sc = -INFINITY;
    if (keep) {
      const int64_t kr = int64_t(base + j) * 3 * hd + int64_t(H + h) * D;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot += q[d] * ld(qkv, kr + d);
      if (a.rel) {
        const int64_t pp = a.relidx[int64_t(i) * a.L + j];
        float c2p = 0.f, p2c = 0.f;
        for (int d = 0; d < D; ++d) {
          c2p += q[d] * ld(pk, pp * hd + int64_t(h) * D + d);
          p2c += ld(qkv, kr + d) * ld(pq, pp * hd + int64_t(h) * D + d);
        }
        sc = (dot + c2p + p2c) * a.scale;
      } else {
        sc = dot * a.scale;
      }
    }
    float cmax = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
    if (cmax == -INFINITY) continue;  // no kept key in this chunk
    const float mn = fmaxf(m, cmax);
    const float corr = expf(m - mn);
    const float pe = keep ? expf(sc - mn) : 0.f;
    float psum = pe;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * corr + psum;
    acc0 *= corr;
    acc1 *= corr;
    const int nj = min(32, n - j0);
    for (int jj = 0; jj < nj; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, pe, jj);
      if (pj == 0.f) continue;  // a key not kept (or with no weight): its value row stays out
      const int64_t vr = int64_t(base + j0 + jj) * 3 * hd + int64_t(2 * H + h) * D;
      if (lane < D) acc0 += pj * ld(qkv, vr + lane);
      if (lane + 32 < D) acc1 += pj * ld(qkv, vr + lane + 32);
    }
    m = mn;
  }
  const float invl = (qvalid && l > 0.f) ? 1.0f / l : 0.f;
  if (lane < D) st(ctx, qrow * hd + int64_t(h) * D + lane, acc0 * invl);
  if (lane + 32 < D) st(ctx, qrow * hd + int64_t(h) * D + lane + 32, acc1 * invl);
}

// Attention without relative terms for the plans the tensor-core kernel does not take (f32 plans,
// head dimensions other than 32 / 64): one CTA per (16 query rows of a sequence, head), the keys
// of those rows staged in shared memory KC at a time (K rows padded to D + 1 floats, so the lanes
// of a warp, one key each, read different banks), then per query row (one warp) the scores of
// its keys, an online softmax over the chunks and the weighted sum of the value rows (one output
// column per lane). Same semantics as attention_simt_kernel: masked query rows are zero, masked
// keys and keys outside the window get no weight and their value rows never enter the sum.
constexpr int SA_ROWS = 16;  // query rows of one CTA
constexpr int SA_WARPS = 8;

template <typename T, int KC>
__global__ void __launch_bounds__(SA_WARPS * 32) attention_smem_kernel(AttnArgs a, SeqTable seq) {
  extern __shared__ float sa_smem[];
  const int D = a.D, DP = D + 1;
  float* sK = sa_smem;        // [KC][D + 1]
  float* sV = sK + KC * DP;   // [KC][D]
  float* sQ = sV + KC * D;    // [SA_ROWS][D]
  const int tile = blockIdx.x / (AROWS_TILE / SA_ROWS), sub = blockIdx.x % (AROWS_TILE / SA_ROWS);
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = seq.tiles[2 * tile], n = seq.len[s], base = seq.start[s];
  const int q0 = seq.tiles[2 * tile + 1] + sub * SA_ROWS;
  if (q0 >= n) return;  // (CTA-uniform)
  const int q1 = min(q0 + SA_ROWS, n);
  const int H = a.H, hd = H * D;
  const T* qkv = static_cast<const T*>(a.qkv);
  T* ctx = static_cast<T*>(a.ctx);
  int jlo = 0, jhi = n;  // keys any of the CTA's rows can keep
  if (a.window) {
    jlo = max(0, q0 - a.window);
    jhi = min(n, q1 + a.window);
  }
  for (int e = threadIdx.x; e < SA_ROWS * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    const int i = q0 + r;
    sQ[e] = i < q1 ? ld(qkv, int64_t(base + i) * 3 * hd + int64_t(h) * D + d) : 0.f;
  }
  constexpr int RPW = SA_ROWS / SA_WARPS;  // rows per warp
  float m[RPW], l[RPW], acc0[RPW], acc1[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    m[r] = -3.40282346638528859812e38f;
    l[r] = 0.f;
    acc0[r] = 0.f;
    acc1[r] = 0.f;
  }
  for (int c0 = jlo; c0 < jhi; c0 += KC) {
    const int nk = min(KC, jhi - c0);
    __syncthreads();  // the previous chunk is consumed (and the query rows are staged)
    for (int e = threadIdx.x; e < KC * D; e += blockDim.x) {
      const int jj = e / D, d = e - jj * D;
      float kv = 0.f, vv = 0.f;
      if (jj < nk) {
        const int64_t kr = int64_t(base + c0 + jj) * 3 * hd;
        kv = ld(qkv, kr + int64_t(H + h) * D + d);
        if (a.mask[base + c0 + jj] > 0.5f) vv = ld(qkv, kr + int64_t(2 * H + h) * D + d);
      }
      sK[jj * DP + d] = kv;
      sV[jj * D + d] = vv;  // masked and absent keys: zero rows
    }
    __syncthreads();
    const int nt = (nk + 31) >> 5;  // 32-key groups with keys in them
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int li = warp + r * SA_WARPS, i = q0 + li;
      if (i >= q1 || !(a.mask[base + i] > 0.5f)) continue;  // (warp-uniform)
      float sc[KC / 32];
#pragma unroll
      for (int t = 0; t < KC / 32; ++t) sc[t] = 0.f;
      const float* q = sQ + li * D;
      for (int d = 0; d < D; ++d) {
        const float qd = q[d];
#pragma unroll
        for (int t = 0; t < KC / 32; ++t) sc[t] += qd * sK[(lane + 32 * t) * DP + d];
      }
      float cmax = -INFINITY;
      bool keep[KC / 32];
#pragma unroll
      for (int t = 0; t < KC / 32; ++t) {
        const int jj = lane + 32 * t, j = c0 + jj;
        keep[t] = jj < nk && a.mask[base + min(j, n - 1)] > 0.5f && !(a.window && abs(i - j) > a.window);
        sc[t] = keep[t] ? sc[t] * a.scale : -INFINITY;
        cmax = fmaxf(cmax, sc[t]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
      if (cmax == -INFINITY) continue;  // no kept key in this chunk
      const float mn = fmaxf(m[r], cmax);
      const float corr = expf(m[r] - mn);
      float psum = 0.f;
#pragma unroll
      for (int t = 0; t < KC / 32; ++t) {
        sc[t] = keep[t] ? expf(sc[t] - mn) : 0.f;
        psum += sc[t];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      l[r] = l[r] * corr + psum;
      float a0 = acc0[r] * corr, a1 = acc1[r] * corr;
#pragma unroll
      for (int t = 0; t < KC / 32; ++t) {
        if (t >= nt) break;
        const float* vrow = sV + 32 * t * D;
#pragma unroll 8
        for (int jj = 0; jj < 32; ++jj) {
          const float pj = __shfl_sync(0xffffffffu, sc[t], jj);
          if (lane < D) a0 += pj * vrow[jj * D + lane];
          if (lane + 32 < D) a1 += pj * vrow[jj * D + lane + 32];
        }
      }
      acc0[r] = a0;
      acc1[r] = a1;
      m[r] = mn;
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int li = warp + r * SA_WARPS, i = q0 + li;
    if (i >= q1) continue;
    const int64_t qrow = int64_t(base) + i;
    const bool live = a.mask[qrow] > 0.5f && l[r] > 0.f;
    const float invl = live ? 1.0f / l[r] : 0.f;
    if (lane < D) st(ctx, qrow * hd + int64_t(h) * D + lane, live ? acc0[r] * invl : 0.f);
    if (lane + 32 < D) st(ctx, qrow * hd + int64_t(h) * D + lane + 32, live ? acc1[r] * invl : 0.f);
  }
}

__global__ void f32_to_f16_kernel(const float* src, __half* dst, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}
__global__ void f16_to_f32_kernel(const __half* src, float* dst, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = __half2float(src[i]);
}

inline int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  return int(g < 1 ? 1 : g);
}

}  // namespace

void launch_embln(bool f16, const void* word, const void* pos, const void* typ, const uint32_t* tt, const void* w,
                  const void* b, const float* mask, void* out, int N, int rows, const int32_t* row_pos, int offset,
                  int maxpos, float eps, int maskmul, int posids, cudaStream_t st) {
  if (N > 32 * MAXE) throw std::runtime_error("embln: width above 1024");
  if (rows <= 0) return;
  const int vn = f16 ? 8 : 4;
  if (N % vn == 0 && N / vn <= 32 * MAXV) {
    const int lpr = lanes_per_row(N / vn);
    const int grid = int((int64_t(rows) * lpr + 255) / 256);
#define KH_EMBLN(TT, L)                                                                                         \
  embln_vec_kernel<TT, L><<<grid, 256, 0, st>>>((const TT*)word, (const TT*)pos, (const TT*)typ, tt, (const TT*)w, \
                                                (const TT*)b, mask, (TT*)out, N, rows, row_pos, offset, maxpos, eps, \
                                                maskmul, posids)
    if (f16) {
      if (lpr == 8) KH_EMBLN(__half, 8); else if (lpr == 16) KH_EMBLN(__half, 16); else KH_EMBLN(__half, 32);
    } else {
      if (lpr == 8) KH_EMBLN(float, 8); else if (lpr == 16) KH_EMBLN(float, 16); else KH_EMBLN(float, 32);
    }
#undef KH_EMBLN
    return;
  }
  const int grid = (rows + 7) / 8;
  if (f16)
    embln_kernel<__half><<<grid, 256, 0, st>>>((const __half*)word, (const __half*)pos, (const __half*)typ, tt,
                                               (const __half*)w, (const __half*)b, mask, (__half*)out, N, rows,
                                               row_pos, offset, maxpos, eps, maskmul, posids);
  else
    embln_kernel<float><<<grid, 256, 0, st>>>((const float*)word, (const float*)pos, (const float*)typ, tt,
                                              (const float*)w, (const float*)b, mask, (float*)out, N, rows, row_pos,
                                              offset, maxpos, eps, maskmul, posids);
}

void launch_layernorm(bool f16, const void* a, const void* b, const void* w, const void* bias, const float* mask,
                      void* out, int N, int rows, int mode, float eps, cudaStream_t st) {
  if (N > 32 * MAXE) throw std::runtime_error("layernorm: width above 1024");
  if (rows <= 0) return;
  const int vn = f16 ? 8 : 4;
  if (N % vn == 0 && N / vn <= 32 * MAXV) {
    const int lpr = lanes_per_row(N / vn);
    const int grid = int((int64_t(rows) * lpr + 255) / 256);
#define KH_LN(TT, L)                                                                                            \
  layernorm_vec_kernel<TT, L><<<grid, 256, 0, st>>>((const TT*)a, (const TT*)b, (const TT*)w, (const TT*)bias, mask, \
                                                    (TT*)out, N, rows, mode, eps)
    if (f16) {
      if (lpr == 8) KH_LN(__half, 8); else if (lpr == 16) KH_LN(__half, 16); else KH_LN(__half, 32);
    } else {
      if (lpr == 8) KH_LN(float, 8); else if (lpr == 16) KH_LN(float, 16); else KH_LN(float, 32);
    }
#undef KH_LN
    return;
  }
  const int grid = (rows + 7) / 8;
  if (f16)
    layernorm_kernel<__half><<<grid, 256, 0, st>>>((const __half*)a, (const __half*)b, (const __half*)w,
                                                   (const __half*)bias, mask, (__half*)out, N, rows, mode, eps);
  else
    layernorm_kernel<float><<<grid, 256, 0, st>>>((const float*)a, (const float*)b, (const float*)w,
                                                  (const float*)bias, mask, (float*)out, N, rows, mode, eps);
}

void launch_add(bool f16, void* dst, const void* src, int64_t count, cudaStream_t st) {
  if (count <= 0) return;
  if (f16) add_kernel<__half><<<grid_for(count, 256), 256, 0, st>>>((__half*)dst, (const __half*)src, count);
  else add_kernel<float><<<grid_for(count, 256), 256, 0, st>>>((float*)dst, (const float*)src, count);
}

void launch_add_rows(bool f16, void* dst, const void* src, int N, int rows, const int32_t* row_seq, cudaStream_t st) {
  const int64_t count = int64_t(rows) * N;
  if (count <= 0) return;
  if (f16) add_rows_kernel<__half><<<grid_for(count, 256), 256, 0, st>>>((__half*)dst, (const __half*)src, N, rows, row_seq);
  else add_rows_kernel<float><<<grid_for(count, 256), 256, 0, st>>>((float*)dst, (const float*)src, N, rows, row_seq);
}

void launch_geglu(bool f16, const void* mid, void* gate, int I, int rows, cudaStream_t st) {
  const int64_t n = int64_t(rows) * I;
  if (n <= 0) return;
  if (f16) geglu_kernel<__half><<<grid_for(n, 256), 256, 0, st>>>((const __half*)mid, (__half*)gate, I, rows);
  else geglu_kernel<float><<<grid_for(n, 256), 256, 0, st>>>((const float*)mid, (float*)gate, I, rows);
}

void launch_rope(bool f16, void* qkv, const float* cossin, const int32_t* row_pos, int H, int D, int rows,
                 cudaStream_t st) {
  const int64_t n = int64_t(rows) * H * D;
  if (n <= 0) return;
  if (f16) rope_kernel<__half><<<grid_for(n, 256), 256, 0, st>>>((__half*)qkv, cossin, row_pos, H, D, rows);
  else rope_kernel<float><<<grid_for(n, 256), 256, 0, st>>>((float*)qkv, cossin, row_pos, H, D, rows);
}

void launch_pool(bool f16, const void* x, const float* mask, void* out, int N, int mode, const SeqTable& seq,
                 cudaStream_t st) {
  if (seq.count <= 0) return;
  dim3 grid((N + 127) / 128, seq.count);
  if (f16) pool_kernel<__half><<<grid, 128, 0, st>>>((const __half*)x, mask, (__half*)out, N, mode, seq.start, seq.len);
  else pool_kernel<float><<<grid, 128, 0, st>>>((const float*)x, mask, (float*)out, N, mode, seq.start, seq.len);
}

void launch_gather(bool f16, const void* x, void* out, int D, const SeqTable& seq, const uint32_t* markers, int K,
                   cudaStream_t st) {
  if (seq.count <= 0) return;
  const int grid = seq.count * K;
  if (f16)
    gather_kernel<__half><<<grid, 128, 0, st>>>((const __half*)x, (__half*)out, D, seq.start, seq.len, markers, K,
                                                seq.count);
  else
    gather_kernel<float><<<grid, 128, 0, st>>>((const float*)x, (float*)out, D, seq.start, seq.len, markers, K,
                                               seq.count);
}

void launch_masklogits(bool f16, const void* raw, const uint32_t* packed, float* logits, int K, float temp,
                       int n_seqs, cudaStream_t st) {
  const int total = n_seqs * K;
  if (total <= 0) return;
  if (f16)
    masklogits_kernel<__half><<<(total + 127) / 128, 128, 0, st>>>((const __half*)raw, packed, logits, K, temp, total);
  else
    masklogits_kernel<float><<<(total + 127) / 128, 128, 0, st>>>((const float*)raw, packed, logits, K, temp, total);
}

void launch_im2col(bool f16, const void* x, const float* mask, void* out, int N, int KS, int rows, const SeqTable& seq,
                   const int32_t* row_seq, cudaStream_t st) {
  if (rows <= 0) return;
  if (f16)
    im2col_kernel<__half><<<rows, 128, 0, st>>>((const __half*)x, mask, (__half*)out, N, KS, rows, seq.start, seq.len,
                                                row_seq, seq.row_pos);
  else
    im2col_kernel<float><<<rows, 128, 0, st>>>((const float*)x, mask, (float*)out, N, KS, rows, seq.start, seq.len,
                                               row_seq, seq.row_pos);
}

void launch_gemm_simt(bool f16, const void* A, const void* W, const void* bias, void* C, int M, int N, int K, int act,
                      cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  const int64_t tiles64 = int64_t((N + 63) / 64) * ((M + 63) / 64);
  if (tiles64 >= 2 * 148) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    if (f16)
      gemm_simt_kernel<__half, 64><<<grid, 256, 0, st>>>((const __half*)A, (const __half*)W, (const __half*)bias,
                                                         (__half*)C, M, N, K, act);
    else
      gemm_simt_kernel<float, 64><<<grid, 256, 0, st>>>((const float*)A, (const float*)W, (const float*)bias,
                                                        (float*)C, M, N, K, act);
  } else {  // small launches (B = 1 calls): four times the CTAs
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    if (f16)
      gemm_simt_kernel<__half, 32><<<grid, 256, 0, st>>>((const __half*)A, (const __half*)W, (const __half*)bias,
                                                         (__half*)C, M, N, K, act);
    else
      gemm_simt_kernel<float, 32><<<grid, 256, 0, st>>>((const float*)A, (const float*)W, (const float*)bias,
                                                        (float*)C, M, N, K, act);
  }
}

void launch_attention_simt(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st) {
  if (a.D > 64) throw std::runtime_error("attention: head dimension above 64");
  if (seq.ntiles <= 0) return;
  if (!a.rel) {
    // keys staged in shared memory: 128 per chunk up to D = 32, else 64 (at most 37 KB)
    dim3 grid(seq.ntiles * (AROWS_TILE / SA_ROWS), a.H);
    const int kc = a.D <= 32 ? 128 : 64;
    const size_t smem = size_t(kc * (a.D + 1) + kc * a.D + SA_ROWS * a.D) * 4;
    if (kc == 128) {
      if (f16) attention_smem_kernel<__half, 128><<<grid, SA_WARPS * 32, smem, st>>>(a, seq);
      else attention_smem_kernel<float, 128><<<grid, SA_WARPS * 32, smem, st>>>(a, seq);
    } else {
      if (f16) attention_smem_kernel<__half, 64><<<grid, SA_WARPS * 32, smem, st>>>(a, seq);
      else attention_smem_kernel<float, 64><<<grid, SA_WARPS * 32, smem, st>>>(a, seq);
    }
    return;
  }
  dim3 grid(seq.ntiles * (AROWS_TILE / AW), a.H);
  if (f16) attention_simt_kernel<__half><<<grid, AW * 32, 0, st>>>(a, seq);
  else attention_simt_kernel<float><<<grid, AW * 32, 0, st>>>(a, seq);
}

void launch_f32_to_f16(const float* src, __half* dst, int64_t n, cudaStream_t st) {
  if (n > 0) f32_to_f16_kernel<<<grid_for(n, 256), 256, 0, st>>>(src, dst, n);
}
void launch_f16_to_f32(const __half* src, float* dst, int64_t n, cudaStream_t st) {
  if (n > 0) f16_to_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(src, dst, n);
}

namespace {
__device__ int kh_gather_bad = 0;

// One warp per row, 16-byte copies (E * element size is a multiple of 16 bytes).
__global__ void gather_rows_kernel(const uint4* __restrict__ table, int64_t vocab, const int32_t* __restrict__ ids,
                                   int64_t n, int row_vecs, uint4* __restrict__ out) {
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const int32_t id = ids[row];
  const bool ok = id >= 0 && int64_t(id) < vocab;
  if (!ok && lane == 0) atomicAdd(&kh_gather_bad, 1);
  const uint4* src = table + int64_t(ok ? id : 0) * row_vecs;
  uint4* dst = out + row * row_vecs;
  for (int v = lane; v < row_vecs; v += 32) dst[v] = ok ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
}
}  // namespace

void launch_gather_rows(bool f16, const void* table, int64_t vocab, const int32_t* ids, int64_t n, int E, void* out,
                        cudaStream_t st) {
  if (n <= 0) return;
  const int64_t row_bytes = int64_t(E) * (f16 ? 2 : 4);
  if (row_bytes % 16) throw PlanError("word rows must be a multiple of 16 bytes");
  const int64_t threads = n * 32;
  gather_rows_kernel<<<unsigned((threads + 255) / 256), 256, 0, st>>>(
      static_cast<const uint4*>(table), vocab, ids, n, int(row_bytes / 16), static_cast<uint4*>(out));
  KH_CUDA(cudaGetLastError());
}

int gather_error_code() {
  int v = 0;
  KH_CUDA(cudaMemcpyFromSymbol(&v, kh_gather_bad, sizeof(int)));
  if (v) {
    const int zero = 0;
    KH_CUDA(cudaMemcpyToSymbol(kh_gather_bad, &zero, sizeof(int)));
  }
  return v;
}

namespace {
// One CTA per chunk: sequence starts and lengths, and the attention work tiles (seq, q0), from an
// exclusive scan of the lengths and of the tiles per sequence.
__global__ void seqtable_chunk_kernel(const int32_t* __restrict__ lens, const ChunkDesc* __restrict__ chunks,
                                      int tile_q, int32_t* __restrict__ table) {
  __shared__ int32_t part_len[1024], part_tiles[1024];
  const ChunkDesc c = chunks[blockIdx.x];
  int32_t* start = table + c.word0;
  int32_t* len = start + c.S;
  int32_t* tiles = len + c.S + 2 * int64_t(c.T);
  const int per = (c.S + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  int32_t sl = 0, st = 0;
  for (int i = 0; i < per; ++i)
    if (b0 + i < c.S) {
      const int32_t l = lens[c.seq0 + b0 + i];
      sl += l;
      st += (l + tile_q - 1) / tile_q;
    }
  part_len[threadIdx.x] = sl;
  part_tiles[threadIdx.x] = st;
  __syncthreads();
  for (int off = 1; off < int(blockDim.x); off <<= 1) {
    const int32_t a = int(threadIdx.x) >= off ? part_len[threadIdx.x - off] : 0;
    const int32_t b = int(threadIdx.x) >= off ? part_tiles[threadIdx.x - off] : 0;
    __syncthreads();
    part_len[threadIdx.x] += a;
    part_tiles[threadIdx.x] += b;
    __syncthreads();
  }
  int32_t rl = part_len[threadIdx.x] - sl, rt = part_tiles[threadIdx.x] - st;
  for (int i = 0; i < per; ++i)
    if (b0 + i < c.S) {
      const int s = b0 + i;
      const int32_t l = lens[c.seq0 + s];
      start[s] = rl;
      len[s] = l;
      for (int q = 0; q < l; q += tile_q) {
        tiles[2 * rt] = s;
        tiles[2 * rt + 1] = q;
        ++rt;
      }
      rl += l;
    }
}

// Thread per packed row of the whole bulk: its chunk, sequence and local position, and for the
// first row of every 128-row tile the tile's key range.
__global__ void seqtable_rows_kernel(const ChunkDesc* __restrict__ chunks, int n_chunks, int64_t total_rows,
                                     int32_t* __restrict__ table) {
  const int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= total_rows) return;
  int lo = 0, hi = n_chunks - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunks[mid].tok0 <= g) lo = mid;
    else hi = mid - 1;
  }
  const ChunkDesc c = chunks[lo];
  const int r = int(g - c.tok0);
  const int32_t* start = table + c.word0;
  const int32_t* len = start + c.S;
  int32_t* pos = table + c.word0 + 2 * int64_t(c.S);
  int32_t* rseq = pos + c.T;
  int32_t* ptiles = rseq + c.T + 2 * int64_t(c.ntiles);
  auto seq_of = [&](int row) {
    int a = 0, b = c.S - 1;  // lengths >= 1: starts strictly increase
    while (a < b) {
      const int mid = (a + b + 1) >> 1;
      if (start[mid] <= row) a = mid;
      else b = mid - 1;
    }
    return a;
  };
  const int s = seq_of(r);
  pos[r] = r - start[s];
  rseq[r] = s;
  if (r % PACKED_TILE == 0) {
    const int s1 = seq_of(min(c.T, r + PACKED_TILE) - 1);
    int32_t* pt = ptiles + 3 * (r / PACKED_TILE);
    pt[0] = r;
    pt[1] = start[s];
    pt[2] = start[s1] + len[s1];
  }
}
}  // namespace

void launch_build_seq_tables(const int32_t* lens, const ChunkDesc* chunks, int n_chunks, int64_t total_rows,
                             int tile_q, int32_t* table, cudaStream_t st) {
  if (n_chunks <= 0 || total_rows <= 0) return;
  seqtable_chunk_kernel<<<n_chunks, 1024, 0, st>>>(lens, chunks, tile_q, table);
  seqtable_rows_kernel<<<unsigned((total_rows + 255) / 256), 256, 0, st>>>(chunks, n_chunks, total_rows, table);
  KH_CUDA(cudaGetLastError());
}

}  // namespace kh
