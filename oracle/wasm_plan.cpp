// ORACLE — test infrastructure only. Not part of the product and never linked into it: only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this library, and only
// as the checker / the timed CPU baseline.
//
// C++ restatement of kleinhirn's WASM-SIMD CPU executor, src/wasm/plan.ts (AssemblyScript,
// compiled to WebAssembly SIMD in the reference). Same op records, same arithmetic, same
// 4-lane accumulation orders: v128 values become GCC vector types of four floats, every
// f32x4 mul/add stays a separate rounding (the file is built with -ffp-contract=off, which is
// the "plain" build of the reference, src/wasm/plan.ts:232-238), horizontal sums add lanes
// 0+1+2+3 left to right (src/wasm/plan.ts:52-55).
//
// Memory model: one byte arena stands in for the WebAssembly linear memory. Addresses in the
// op stream are u32 byte offsets into it, written by the host translation in oracle/host.py
// (the restatement of src/plan/wasm.ts). The arena is grown by the host; this file allocates
// nothing (as src/wasm/plan.ts:7 says of the module).
//
// Scalar stdlib calls: AssemblyScript's Mathf.exp / Mathf.tanh / Mathf.sqrt become libm expf /
// tanhf / sqrtf. Their last bits may differ from AssemblyScript's own implementations; no
// reference test pins bits at that boundary (tests/wasm_plan.test.ts pins 2e-5 relative).
//
// Threads (src/wasm/plan.ts:942-1085): the same work items (rb x cb matmul tiles, 16-row LN
// blocks, 8-row GeGLU blocks, (sequence, head, query block) attention items) claimed from an
// atomic counter by std::thread helpers; every output element is computed by one thread with
// the serial code, so results do not depend on the thread count.

#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

typedef float f4 __attribute__((vector_size(16)));
typedef int32_t i4 __attribute__((vector_size(16)));

namespace {

const int HEAD = 8;   // src/wasm/plan.ts:16
const int OPW = 32;   // src/wasm/plan.ts:17
enum {
  GEMM_P = 1, GEMM_NT = 2, LN = 3, EMBLN = 4, ADD = 5, GATHER = 6, POOL = 7, GEGLU = 8, ROPE = 9,
  IM2COL = 10, ATTSCORE = 11, ATTSOFTMAX = 12, ATTPV = 13, ATTREL = 14, ATTSOFTREL = 15, ATTSTD = 16,
  ATTRELF = 17, MASKLOGITS = 18,
};
const float LOWEST = -3.40282346638528859812e38f;  // src/wasm/plan.ts:38-39

uint8_t* MEM = nullptr;  // the arena of the current run

inline float* fp(uint32_t p) { return reinterpret_cast<float*>(MEM + p); }
inline int32_t* ip(uint32_t p) { return reinterpret_cast<int32_t*>(MEM + p); }
inline float ldf(uint32_t p, int i) { return fp(p)[i]; }
inline void stf(uint32_t p, int i, float v) { fp(p)[i] = v; }
inline int32_t ldi(uint32_t p, int i) { return ip(p)[i]; }
inline uint32_t off(uint32_t p, int i) { return p + (uint32_t(i) << 2); }
inline f4 vld(uint32_t p) { f4 v; std::memcpy(&v, MEM + p, 16); return v; }
inline void vst(uint32_t p, f4 v) { std::memcpy(MEM + p, &v, 16); }
inline f4 splat(float x) { return f4{x, x, x, x}; }
inline float hsum(f4 v) { return v[0] + v[1] + v[2] + v[3]; }
// WebAssembly f32.min / f32.max (and their f32x4 lanes, which AssemblyScript's Mathf.min / max
// and f32x4.min / max compile to): a NaN operand gives NaN, and -0 < +0. std::fmin / fmax would
// return the other operand for a NaN.
// (selects, not branches: the compiler keeps the lanes in vector registers)
inline float wmin(float a, float b) {
  float r = a < b ? a : b;
  r = a == b ? (std::signbit(a) ? a : b) : r;
  return (a != a || b != b) ? a + b : r;  // a NaN operand: NaN
}
inline float wmax(float a, float b) {
  float r = a > b ? a : b;
  r = a == b ? (std::signbit(a) ? b : a) : r;
  return (a != a || b != b) ? a + b : r;  // a NaN operand: NaN
}
inline f4 vmin(f4 a, f4 b) { return f4{wmin(a[0], b[0]), wmin(a[1], b[1]), wmin(a[2], b[2]), wmin(a[3], b[3])}; }
inline f4 vmax(f4 a, f4 b) { return f4{wmax(a[0], b[0]), wmax(a[1], b[1]), wmax(a[2], b[2]), wmax(a[3], b[3])}; }
inline f4 vfloor(f4 a) { return f4{std::floor(a[0]), std::floor(a[1]), std::floor(a[2]), std::floor(a[3])}; }
inline f4 vabs(f4 a) { return f4{std::fabs(a[0]), std::fabs(a[1]), std::fabs(a[2]), std::fabs(a[3])}; }
inline int32_t truncsat(float x) {
  if (std::isnan(x)) return 0;
  if (x >= 2147483647.0f) return 2147483647;
  if (x <= -2147483648.0f) return INT32_MIN;
  return int32_t(x);
}

// src/wasm/plan.ts:61-75: Cephes expf minimax on four lanes, 2^n through the exponent bits.
inline f4 vexp(f4 x) {
  x = vmax(vmin(x, splat(88.3762626647949f)), splat(-87.3365447504f));
  const f4 n = vfloor(x * splat(1.44269504088896341f) + splat(0.5f));
  f4 r = x - n * splat(0.693359375f);
  r = r - n * splat(-2.12194440e-4f);
  f4 y = splat(1.9875691500e-4f);
  y = y * r + splat(1.3981999507e-3f);
  y = y * r + splat(8.3334519073e-3f);
  y = y * r + splat(4.1665795894e-2f);
  y = y * r + splat(1.6666665459e-1f);
  y = y * r + splat(5.0000001201e-1f);
  y = ((y * r) * r + r) + splat(1.0f);
  i4 ni = i4{truncsat(n[0]), truncsat(n[1]), truncsat(n[2]), truncsat(n[3])};
  i4 bits = (ni + i4{127, 127, 127, 127}) << 23;
  f4 pow2n;
  std::memcpy(&pow2n, &bits, 16);
  return y * pow2n;
}
inline float vexp1(float x) { return vexp(splat(x))[0]; }

// src/wasm/plan.ts:82-93: GELU with the A&S 7.1.26 erf on four lanes.
inline f4 vgelu(f4 v) {
  const f4 u = v * splat(0.7071067811865476f);
  const f4 t = splat(1.0f) / (splat(1.0f) + splat(0.3275911f) * vabs(u));
  f4 p = splat(1.061405429f) * t - splat(1.453152027f);
  p = p * t + splat(1.421413741f);
  p = p * t - splat(0.284496736f);
  p = p * t + splat(0.254829592f);
  p = p * t;
  const f4 e = splat(1.0f) - p * vexp(-(u * u));
  f4 se;
  for (int l = 0; l < 4; ++l) se[l] = v[l] >= 0 ? e[l] : -e[l];
  return (splat(0.5f) * v) * (splat(1.0f) + se);
}
inline float vgelu1(float v) { return vgelu(splat(v))[0]; }

// src/wasm/plan.ts:100-107
inline float gelu(float v) {
  const float u = v * 0.7071067811865476f;
  const float t = 1.0f / (1.0f + 0.3275911f * std::fabs(u));
  const float p = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
  const float e = 1.0f - p * expf(-u * u);
  return 0.5f * v * (1.0f + (v >= 0 ? e : -e));
}

// src/wasm/plan.ts:110-116
float activate(float v, int act) {
  if (act == 1) return wmax(v, 0.0f);
  if (act == 2) return gelu(v);
  if (act == 3) return tanhf(v);
  if (act == 4) return v / (1.0f + expf(-v));
  return v;
}

inline float fin(float acc, float alpha, uint32_t bias, int n, int act) {
  float v = acc * alpha;
  if (bias) v += ldf(bias, n);
  return act ? activate(v, act) : v;
}

// src/wasm/plan.ts:130-154
void biasAct(uint32_t c, int ldc, uint32_t bias, int M, int N, int act) {
  for (int m = 0; m < M; ++m) {
    const uint32_t r = off(c, m * ldc);
    int n0 = 0;
    if (act == 2 || act == 0) {
      for (; n0 + 4 <= N; n0 += 4) {
        f4 v = vld(off(r, n0));
        if (bias) v = v + vld(off(bias, n0));
        vst(off(r, n0), act ? vgelu(v) : v);
      }
      for (; n0 < N; ++n0) {
        float v = ldf(r, n0);
        if (bias) v += ldf(bias, n0);
        stf(r, n0, act ? vgelu1(v) : v);
      }
      continue;
    }
    for (int n = 0; n < N; ++n) {
      float v = ldf(r, n);
      if (bias) v += ldf(bias, n);
      stf(r, n, act ? activate(v, act) : v);
    }
  }
}

inline void storeAcc(uint32_t c, f4 acc, int take) {
  if (take >= 4) { vst(c, acc); return; }
  if (take >= 1) stf(c, 0, acc[0]);
  if (take >= 2) stf(c, 1, acc[1]);
  if (take >= 3) stf(c, 2, acc[2]);
}

inline void storeRow(uint32_t c, int lanes, f4 a0, f4 a1, f4 a2, f4 a3) {
  storeAcc(c, a0, lanes);
  storeAcc(c + 16, a1, lanes - 4);
  storeAcc(c + 32, a2, lanes - 8);
  storeAcc(c + 48, a3, lanes - 12);
}

// src/wasm/plan.ts:235-238 (plain build: mul, then add)
inline f4 madd(f4 x, f4 w, f4 acc) { return (x * w) + acc; }

// src/wasm/plan.ts:174-230
void gemmNN(uint32_t a, int lda, uint32_t b, int ldb, uint32_t c, int ldc, int M, int N, int K) {
  const uint32_t sa = uint32_t(lda) << 2;
  for (int mb = 0; mb < M; mb += 4) {
    const int rows = std::min(M - mb, 4);
    const uint32_t aRow = a + (uint32_t(mb * lda) << 2);
    for (int nb = 0; nb < N; nb += 16) {
      f4 z = splat(0);
      f4 a00 = z, a01 = z, a02 = z, a03 = z, a10 = z, a11 = z, a12 = z, a13 = z;
      f4 a20 = z, a21 = z, a22 = z, a23 = z, a30 = z, a31 = z, a32 = z, a33 = z;
      uint32_t bp = b + (uint32_t(nb) << 2);
      const uint32_t sb = uint32_t(ldb) << 2;
      for (int k = 0; k < K; ++k) {
        const f4 w0 = vld(bp), w1 = vld(bp + 16), w2 = vld(bp + 32), w3 = vld(bp + 48);
        bp += sb;
        const uint32_t ap = aRow + (uint32_t(k) << 2);
        const f4 v0 = splat(*fp(ap));
        a00 = madd(v0, w0, a00); a01 = madd(v0, w1, a01); a02 = madd(v0, w2, a02); a03 = madd(v0, w3, a03);
        if (rows >= 2) {
          const f4 v1 = splat(*fp(ap + sa));
          a10 = madd(v1, w0, a10); a11 = madd(v1, w1, a11); a12 = madd(v1, w2, a12); a13 = madd(v1, w3, a13);
          if (rows >= 3) {
            const f4 v2 = splat(*fp(ap + 2 * sa));
            a20 = madd(v2, w0, a20); a21 = madd(v2, w1, a21); a22 = madd(v2, w2, a22); a23 = madd(v2, w3, a23);
            if (rows >= 4) {
              const f4 v3 = splat(*fp(ap + 3 * sa));
              a30 = madd(v3, w0, a30); a31 = madd(v3, w1, a31); a32 = madd(v3, w2, a32); a33 = madd(v3, w3, a33);
            }
          }
        }
      }
      const int lanes = std::min(N - nb, 16);
      const uint32_t c0 = c + (uint32_t(mb * ldc + nb) << 2);
      const uint32_t sc = uint32_t(ldc) << 2;
      storeRow(c0, lanes, a00, a01, a02, a03);
      if (rows >= 2) storeRow(c0 + sc, lanes, a10, a11, a12, a13);
      if (rows >= 3) storeRow(c0 + 2 * sc, lanes, a20, a21, a22, a23);
      if (rows >= 4) storeRow(c0 + 3 * sc, lanes, a30, a31, a32, a33);
    }
  }
}

// src/wasm/plan.ts:244-295: B in panels [ceil(N / 16)][K][16]
void gemmP(uint32_t a, int lda, uint32_t p, uint32_t c, int ldc, int M, int N, int K) {
  const uint32_t sa = uint32_t(lda) << 2;
  const uint32_t sc = uint32_t(ldc) << 2;
  const uint32_t ps = uint32_t(K) << 6;
  int m = 0;
  for (; m + 4 <= M; m += 4) {
    const uint32_t ar = a + uint32_t(m) * sa;
    for (int nb = 0; nb < N; nb += 16) {
      f4 z = splat(0);
      f4 a00 = z, a01 = z, a02 = z, a03 = z, a10 = z, a11 = z, a12 = z, a13 = z;
      f4 a20 = z, a21 = z, a22 = z, a23 = z, a30 = z, a31 = z, a32 = z, a33 = z;
      uint32_t bp = p + uint32_t(nb >> 4) * ps;
      for (int k = 0; k < K; ++k) {
        const f4 w0 = vld(bp), w1 = vld(bp + 16), w2 = vld(bp + 32), w3 = vld(bp + 48);
        bp += 64;
        const uint32_t q = ar + (uint32_t(k) << 2);
        const f4 x0 = splat(*fp(q));
        a00 = madd(x0, w0, a00); a01 = madd(x0, w1, a01); a02 = madd(x0, w2, a02); a03 = madd(x0, w3, a03);
        const f4 x1 = splat(*fp(q + sa));
        a10 = madd(x1, w0, a10); a11 = madd(x1, w1, a11); a12 = madd(x1, w2, a12); a13 = madd(x1, w3, a13);
        const f4 x2 = splat(*fp(q + 2 * sa));
        a20 = madd(x2, w0, a20); a21 = madd(x2, w1, a21); a22 = madd(x2, w2, a22); a23 = madd(x2, w3, a23);
        const f4 x3 = splat(*fp(q + 3 * sa));
        a30 = madd(x3, w0, a30); a31 = madd(x3, w1, a31); a32 = madd(x3, w2, a32); a33 = madd(x3, w3, a33);
      }
      const int lanes = std::min(N - nb, 16);
      const uint32_t c0 = c + uint32_t(m) * sc + (uint32_t(nb) << 2);
      storeRow(c0, lanes, a00, a01, a02, a03);
      storeRow(c0 + sc, lanes, a10, a11, a12, a13);
      storeRow(c0 + 2 * sc, lanes, a20, a21, a22, a23);
      storeRow(c0 + 3 * sc, lanes, a30, a31, a32, a33);
    }
  }
  for (; m < M; ++m) {
    const uint32_t ar = a + uint32_t(m) * sa;
    for (int nb = 0; nb < N; nb += 16) {
      f4 s0 = splat(0), s1 = s0, s2 = s0, s3 = s0;
      uint32_t bp = p + uint32_t(nb >> 4) * ps;
      for (int k = 0; k < K; ++k) {
        const f4 x = splat(*fp(ar + (uint32_t(k) << 2)));
        s0 = madd(x, vld(bp), s0); s1 = madd(x, vld(bp + 16), s1);
        s2 = madd(x, vld(bp + 32), s2); s3 = madd(x, vld(bp + 48), s3);
        bp += 64;
      }
      storeRow(c + uint32_t(m) * sc + (uint32_t(nb) << 2), std::min(N - nb, 16), s0, s1, s2, s3);
    }
  }
}

// src/wasm/plan.ts:298-307
float dot(uint32_t a, uint32_t w, int K) {
  f4 acc = splat(0);
  int k = 0;
  for (; k + 4 <= K; k += 4) acc = acc + vld(off(a, k)) * vld(off(w, k));
  float s = hsum(acc);
  for (; k < K; ++k) s += ldf(a, k) * ldf(w, k);
  return s;
}

inline float tailsum(uint32_t x, uint32_t y, int k0, int K) {
  float s = 0;
  for (int k = k0; k < K; ++k) s += ldf(x, k) * ldf(y, k);
  return s;
}

inline void ntStore(uint32_t o, uint32_t x, uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3, int K4, int K,
                    f4 v0, f4 v1, f4 v2, f4 v3, float alpha, uint32_t bias, int n, int act) {
  stf(o, 0, fin(hsum(v0) + tailsum(x, q0, K4, K), alpha, bias, n, act));
  stf(o, 1, fin(hsum(v1) + tailsum(x, q1, K4, K), alpha, bias, n + 1, act));
  stf(o, 2, fin(hsum(v2) + tailsum(x, q2, K4, K), alpha, bias, n + 2, act));
  stf(o, 3, fin(hsum(v3) + tailsum(x, q3, K4, K), alpha, bias, n + 3, act));
}

// src/wasm/plan.ts:311-368
void gemmNT(uint32_t a, int lda, uint32_t b, int ldb, uint32_t c, int ldc, uint32_t bias,
            int M, int N, int K, float alpha, int act) {
  const int K4 = K & ~3;
  int m = 0;
  for (; m + 4 <= M; m += 4) {
    const uint32_t r0 = a + (uint32_t(m * lda) << 2);
    const uint32_t r1 = r0 + (uint32_t(lda) << 2);
    const uint32_t r2 = r1 + (uint32_t(lda) << 2);
    const uint32_t r3 = r2 + (uint32_t(lda) << 2);
    int n = 0;
    for (; n + 4 <= N; n += 4) {
      const uint32_t q0 = b + (uint32_t(n * ldb) << 2);
      const uint32_t q1 = q0 + (uint32_t(ldb) << 2);
      const uint32_t q2 = q1 + (uint32_t(ldb) << 2);
      const uint32_t q3 = q2 + (uint32_t(ldb) << 2);
      f4 z = splat(0);
      f4 c00 = z, c01 = z, c02 = z, c03 = z, c10 = z, c11 = z, c12 = z, c13 = z;
      f4 c20 = z, c21 = z, c22 = z, c23 = z, c30 = z, c31 = z, c32 = z, c33 = z;
      for (int k = 0; k < K4; k += 4) {
        const uint32_t o = uint32_t(k) << 2;
        const f4 x0 = vld(r0 + o), x1 = vld(r1 + o), x2 = vld(r2 + o), x3 = vld(r3 + o);
        const f4 y0 = vld(q0 + o), y1 = vld(q1 + o), y2 = vld(q2 + o), y3 = vld(q3 + o);
        c00 = c00 + x0 * y0; c01 = c01 + x0 * y1; c02 = c02 + x0 * y2; c03 = c03 + x0 * y3;
        c10 = c10 + x1 * y0; c11 = c11 + x1 * y1; c12 = c12 + x1 * y2; c13 = c13 + x1 * y3;
        c20 = c20 + x2 * y0; c21 = c21 + x2 * y1; c22 = c22 + x2 * y2; c23 = c23 + x2 * y3;
        c30 = c30 + x3 * y0; c31 = c31 + x3 * y1; c32 = c32 + x3 * y2; c33 = c33 + x3 * y3;
      }
      const uint32_t o0 = c + (uint32_t(m * ldc + n) << 2);
      const uint32_t sc = uint32_t(ldc) << 2;
      ntStore(o0, r0, q0, q1, q2, q3, K4, K, c00, c01, c02, c03, alpha, bias, n, act);
      ntStore(o0 + sc, r1, q0, q1, q2, q3, K4, K, c10, c11, c12, c13, alpha, bias, n, act);
      ntStore(o0 + 2 * sc, r2, q0, q1, q2, q3, K4, K, c20, c21, c22, c23, alpha, bias, n, act);
      ntStore(o0 + 3 * sc, r3, q0, q1, q2, q3, K4, K, c30, c31, c32, c33, alpha, bias, n, act);
    }
    for (; n < N; ++n) {
      const uint32_t q = b + (uint32_t(n * ldb) << 2);
      const uint32_t o0 = c + (uint32_t(m * ldc + n) << 2);
      const uint32_t sc = uint32_t(ldc) << 2;
      *fp(o0) = fin(dot(r0, q, K), alpha, bias, n, act);
      *fp(o0 + sc) = fin(dot(r1, q, K), alpha, bias, n, act);
      *fp(o0 + 2 * sc) = fin(dot(r2, q, K), alpha, bias, n, act);
      *fp(o0 + 3 * sc) = fin(dot(r3, q, K), alpha, bias, n, act);
    }
  }
  for (; m < M; ++m) {
    const uint32_t r = a + (uint32_t(m * lda) << 2);
    for (int n = 0; n < N; ++n) stf(c, m * ldc + n, fin(dot(r, b + (uint32_t(n * ldb) << 2), K), alpha, bias, n, act));
  }
}

// src/wasm/plan.ts:388-411: two-pass LayerNorm of row o in place
void normRow(uint32_t o, int N, uint32_t w, uint32_t bias, float eps, float scale) {
  f4 acc = splat(0);
  int d = 0;
  for (; d + 4 <= N; d += 4) acc = acc + vld(off(o, d));
  float s = hsum(acc);
  for (; d < N; ++d) s += ldf(o, d);
  const float mean = s / float(N);
  const f4 mv = splat(mean);
  acc = splat(0);
  d = 0;
  for (; d + 4 <= N; d += 4) {
    const f4 x = vld(off(o, d)) - mv;
    acc = acc + x * x;
  }
  float sq = hsum(acc);
  for (; d < N; ++d) {
    const float x = ldf(o, d) - mean;
    sq += x * x;
  }
  const float inv = 1.0f / sqrtf(sq / float(N) + eps);
  for (d = 0; d < N; ++d) stf(o, d, ((ldf(o, d) - mean) * inv * ldf(w, d) + ldf(bias, d)) * scale);
}

// src/wasm/plan.ts:414-431
void layernorm(uint32_t a, uint32_t b, uint32_t w, uint32_t bias, uint32_t mask, uint32_t out,
               int N, int mode, float eps, int r0, int r1) {
  for (int r = r0; r < r1; ++r) {
    const uint32_t o = off(out, r * N);
    const uint32_t x = off(a, r * N);
    if (mode == 2) {
      const uint32_t y = off(b, r * N);
      int d = 0;
      for (; d + 4 <= N; d += 4) vst(off(o, d), vld(off(x, d)) + vld(off(y, d)));
      for (; d < N; ++d) stf(o, d, ldf(x, d) + ldf(y, d));
    } else {
      std::memmove(MEM + o, MEM + x, size_t(N) << 2);
    }
    normRow(o, N, w, bias, eps, mode == 1 ? ldf(mask, r) : 1.0f);
  }
}

// src/wasm/plan.ts:434-447
void embln(uint32_t word, uint32_t pos, uint32_t typ, uint32_t tt, uint32_t w, uint32_t bias, uint32_t mask,
           uint32_t out, int N, int L, int offset, int maxpos, float eps, int maskmul, int posids, int rows) {
  for (int r = 0; r < rows; ++r) {
    const uint32_t t = uint32_t(ldi(tt, r));
    const int prow = posids ? int(t >> 16) : (r % L) + offset;
    const uint32_t p = off(pos, std::min(prow, maxpos - 1) * N);
    const uint32_t y = off(typ, int(t & 0xffff) * N);
    const uint32_t x = off(word, r * N);
    const uint32_t o = off(out, r * N);
    for (int d = 0; d < N; ++d) stf(o, d, ldf(x, d) + ldf(p, d) + ldf(y, d));
    normRow(o, N, w, bias, eps, maskmul ? ldf(mask, r) : 1.0f);
  }
}

// src/wasm/plan.ts:452-464
void add(uint32_t dst, uint32_t src, int count, int N, int mode, int L) {
  if (mode == 0) {
    int i = 0;
    for (; i + 4 <= count; i += 4) vst(off(dst, i), vld(off(dst, i)) + vld(off(src, i)));
    for (; i < count; ++i) stf(dst, i, ldf(dst, i) + ldf(src, i));
    return;
  }
  for (int i = 0; i < count; ++i) stf(dst, i, ldf(dst, i) + ldf(src, (i / (N * L)) * N + i % N));
}

// src/wasm/plan.ts:466-472
void gather(uint32_t markers, uint32_t x, uint32_t states, int K, int D, int L, int total) {
  for (int g = 0; g < total; ++g) {
    const int b = g / K;
    const int row = b * L + ldi(markers, b * 3 * K + (g - b * K));
    std::memmove(MEM + off(states, g * D), MEM + off(x, row * D), size_t(D) << 2);
  }
}

// src/wasm/plan.ts:475-498
void pool(uint32_t x, uint32_t mask, uint32_t out, int L, int N, int mode, int batch) {
  for (int b = 0; b < batch; ++b) {
    const uint32_t o = off(out, b * N);
    for (int d = 0; d < N; ++d) stf(o, d, 0);
    float cnt = 0;
    bool found = false;
    for (int i = 0; i < L; ++i) {
      const float m = ldf(mask, b * L + i);
      const uint32_t xr = off(x, (b * L + i) * N);
      if (mode == 0) {
        if (m == 0) continue;
        for (int d = 0; d < N; ++d) stf(o, d, ldf(o, d) + m * ldf(xr, d));
        cnt += m;
      } else if (m > 0.5f) {
        for (int d = 0; d < N; ++d) stf(o, d, found ? wmax(ldf(o, d), ldf(xr, d)) : ldf(xr, d));
        found = true;
      }
    }
    if (mode == 0) {
      const float den = wmax(cnt, 1e-9f);
      for (int d = 0; d < N; ++d) stf(o, d, ldf(o, d) / den);
    }
  }
}

// src/wasm/plan.ts:500-508
void geglu(uint32_t mid, uint32_t gate, int I, int r0, int r1) {
  for (int r = r0; r < r1; ++r) {
    const uint32_t m = off(mid, r * 2 * I);
    const uint32_t g = off(gate, r * I);
    int j = 0;
    for (; j + 4 <= I; j += 4) vst(off(g, j), vgelu(vld(off(m, j))) * vld(off(m, I + j)));
    for (; j < I; ++j) stf(g, j, vgelu1(ldf(m, j)) * ldf(m, I + j));
  }
}

// src/wasm/plan.ts:511-528
void rope(uint32_t qkv, uint32_t cossin, int L, int H, int D, int rows) {
  const int hd = H * D;
  const int half = D / 2;
  for (int i = 0; i < rows; ++i) {
    const uint32_t t = off(cossin, (i % L) * 2 * D);
    for (int s = 0; s < 2 * H; ++s) {
      const uint32_t base = off(qkv, i * 3 * hd + s * D);
      for (int d = 0; d < half; ++d) {
        const float x = ldf(base, d), y = ldf(base, d + half);
        const float c = ldf(t, d), sn = ldf(t, D + d);
        stf(base, d, x * c - y * sn);
        stf(base, d + half, y * c + x * sn);
      }
    }
  }
}

// src/wasm/plan.ts:530-543
void im2col(uint32_t emb, uint32_t mask, uint32_t out, int N, int L, int KS, int rows) {
  const int pad = (KS - 1) / 2;
  for (int r = 0; r < rows; ++r) {
    const int seq = r / L;
    const int i = r % L;
    for (int t = 0; t < KS; ++t) {
      const int j = i + t - pad;
      const int src = seq * L + std::max(j, 0);
      const uint32_t o = off(out, r * KS * N + t * N);
      if (j >= 0 && j < L && ldf(mask, src) != 0) std::memmove(MEM + o, MEM + off(emb, src * N), size_t(N) << 2);
      else std::memset(MEM + o, 0, size_t(N) << 2);
    }
  }
}

// src/wasm/plan.ts:545-551
void masklogits(uint32_t raw, uint32_t packed, uint32_t logits, int K, float temp, int total) {
  for (int k = 0; k < total; ++k) {
    const int b = k / K;
    const float m = ldf(packed, b * 3 * K + K + (k - b * K));
    stf(logits, k, m > 0.5f ? ldf(raw, k) / temp : -1e4f);
  }
}

// src/wasm/plan.ts:556-569
void keyRanges(uint32_t mask, uint32_t kinfo, int L, int batch) {
  for (int b = 0; b < batch; ++b) {
    int first = L, last = 0;
    for (int j = 0; j < L; ++j) {
      if (ldf(mask, b * L + j) > 0.5f) {
        if (first == L) first = j;
        last = j;
      }
    }
    *ip(kinfo + (uint32_t(2 * b) << 2)) = first;
    *ip(kinfo + (uint32_t(2 * b + 1) << 2)) = last;
  }
}

inline int seqRows(int rows, int b, int L) { return std::min(L, rows - b * L); }

inline bool keep(uint32_t mask, int j, int il, int window) {
  if (ldf(mask, j) <= 0.5f) return false;
  return window == 0 || std::abs(il - j) <= window;
}

// src/wasm/plan.ts:578-634
void softmaxRow(uint32_t p, int n, uint32_t mask, int first, int il, int window, bool qmask, bool dense, float scale) {
  if (!qmask) {
    std::memset(MEM + p, 0, size_t(n) << 2);
    return;
  }
  if (dense) {
    const f4 vsc = splat(scale);
    f4 vm = splat(LOWEST);
    int j = 0;
    for (; j + 4 <= n; j += 4) {
      const f4 x = vld(off(p, j)) * vsc;
      vst(off(p, j), x);
      vm = vmax(vm, x);
    }
    float m = wmax(wmax(vm[0], vm[1]), wmax(vm[2], vm[3]));
    for (; j < n; ++j) {
      const float x = ldf(p, j) * scale;
      stf(p, j, x);
      m = wmax(m, x);
    }
    const f4 vmx = splat(m);
    f4 vs = splat(0);
    j = 0;
    for (; j + 4 <= n; j += 4) {
      const f4 e = vexp(vld(off(p, j)) - vmx);
      vst(off(p, j), e);
      vs = vs + e;
    }
    float s = hsum(vs);
    for (; j < n; ++j) {
      const float e = vexp1(ldf(p, j) - m);
      stf(p, j, e);
      s += e;
    }
    const f4 vi = splat(s > 0 ? 1.0f / s : 0.0f);
    j = 0;
    for (; j + 4 <= n; j += 4) vst(off(p, j), vld(off(p, j)) * vi);
    for (; j < n; ++j) stf(p, j, ldf(p, j) * vi[0]);
    return;
  }
  if (scale != 1) for (int j = 0; j < n; ++j) stf(p, j, ldf(p, j) * scale);
  float mx = LOWEST;
  for (int j = 0; j < n; ++j) if (keep(mask, first + j, il, window)) mx = wmax(mx, ldf(p, j));
  float sum = 0;
  for (int j = 0; j < n; ++j) {
    float e = 0;
    if (keep(mask, first + j, il, window)) e = expf(ldf(p, j) - mx);
    stf(p, j, e);
    sum += e;
  }
  const float inv = sum > 0 ? 1.0f / sum : 0.0f;
  for (int j = 0; j < n; ++j) stf(p, j, ldf(p, j) * inv);
}

// src/wasm/plan.ts:638-650
void packPanels(uint32_t x, int ld, int n, int D, uint32_t out) {
  const int nb = (n + 15) >> 4;
  for (int pb = 0; pb < nb; ++pb) {
    const uint32_t base = off(out, pb * D * 16);
    const int j0 = pb * 16;
    const int lanes = std::min(16, n - j0);
    if (lanes < 16) std::memset(MEM + base, 0, size_t(D * 16) << 2);
    for (int l = 0; l < lanes; ++l) {
      const uint32_t src = off(x, (j0 + l) * ld);
      for (int d = 0; d < D; ++d) stf(base, d * 16 + l, ldf(src, d));
    }
  }
}

// src/wasm/plan.ts:653-656
bool allKeys(uint32_t mask, int first, int last) {
  for (int j = first; j <= last; ++j) if (ldf(mask, j) <= 0.5f) return false;
  return true;
}

// src/wasm/plan.ts:664-679
void attscore(uint32_t qkv, uint32_t scores, uint32_t kinfo, int L, int H, int D, float scale, int rows, int batch) {
  const int hd = H * D;
  for (int b = 0; b < batch; ++b) {
    const int nq = seqRows(rows, b, L);
    const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
    if (nq <= 0 || first >= L) continue;
    for (int h = 0; h < H; ++h) {
      gemmNT(off(qkv, b * L * 3 * hd + h * D), 3 * hd, off(qkv, (b * L + first) * 3 * hd + (H + h) * D), 3 * hd,
             off(scores, (b * L * H + h) * L + first), H * L, 0, nq, last - first + 1, D, scale, 0);
    }
  }
}

// src/wasm/plan.ts:681-694
void attsoftmax(uint32_t mask, uint32_t scores, uint32_t kinfo, int L, int H, int window, int rows) {
  for (int i = 0; i < rows; ++i) {
    const int b = i / L;
    const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
    if (first >= L) continue;
    const uint32_t mk = off(mask, b * L);
    for (int h = 0; h < H; ++h) {
      softmaxRow(off(scores, (i * H + h) * L + first), last - first + 1, mk, first, i - b * L, window,
                 ldf(mask, i) > 0.5f, false, 1);
    }
  }
}

// src/wasm/plan.ts:697-715
void attpv(uint32_t scores, uint32_t qkv, uint32_t ctx, uint32_t kinfo, int L, int H, int D, int rows, int batch) {
  const int hd = H * D;
  for (int b = 0; b < batch; ++b) {
    const int nq = seqRows(rows, b, L);
    if (nq <= 0) continue;
    const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
    if (first >= L) {
      std::memset(MEM + off(ctx, b * L * hd), 0, size_t(nq * hd) << 2);
      continue;
    }
    for (int h = 0; h < H; ++h) {
      gemmNN(off(scores, (b * L * H + h) * L + first), H * L, off(qkv, (b * L + first) * 3 * hd + (2 * H + h) * D),
             3 * hd, off(ctx, b * L * hd + h * D), hd, nq, D, last - first + 1);
    }
  }
}

// src/wasm/plan.ts:719-735
void attrel(uint32_t qkv, uint32_t table, uint32_t relidx, uint32_t out, uint32_t kinfo, int H, int D, int NM,
            int moff, int part, int L, int rows, int batch) {
  const int hd = H * D;
  for (int b = 0; b < batch; ++b) {
    const int nq = seqRows(rows, b, L);
    const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
    if (nq <= 0 || first >= L) continue;
    const int lo = ldi(relidx, first * L + last) - moff;
    const int hi = ldi(relidx, last * L + first) - moff;
    for (int h = 0; h < H; ++h) {
      gemmNT(off(qkv, b * L * 3 * hd + (part * H + h) * D), 3 * hd, off(table, (moff + lo) * hd + h * D), hd,
             off(out, (b * L * H + h) * NM + lo), H * NM, 0, nq, hi - lo + 1, D, 1, 0);
    }
  }
}

// src/wasm/plan.ts:739-762
void attsoftrel(uint32_t mask, uint32_t relidx, uint32_t c2p, uint32_t p2c, uint32_t scores, uint32_t kinfo,
                int L, int H, int NM, int moff, float invscale, int rows) {
  for (int i = 0; i < rows; ++i) {
    const int b = i / L;
    const int il = i - b * L;
    const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
    if (first >= L) continue;
    const bool qm = ldf(mask, i) > 0.5f;
    for (int h = 0; h < H; ++h) {
      const uint32_t p = off(scores, (i * H + h) * L + first);
      if (qm) {
        const uint32_t c = off(c2p, (i * H + h) * NM);
        for (int j = first; j <= last; ++j) {
          if (ldf(mask, b * L + j) <= 0.5f) continue;
          const int m = ldi(relidx, il * L + j) - moff;
          stf(p, j - first, ldf(p, j - first) + (ldf(c, m) + ldf(p2c, ((b * L + j) * H + h) * NM + m)) * invscale);
        }
      }
      softmaxRow(p, last - first + 1, off(mask, b * L), first, il, 0, qm, false, 1);
    }
  }
}

// src/wasm/plan.ts:767-789
void attstdBlock(uint32_t qkv, uint32_t mask, uint32_t ctx, uint32_t kinfo, uint32_t scratch, int L, int H, int D,
                 float scale, int window, int rows, int b, int h, int i0, int i1) {
  const int hd = H * D;
  const int e = std::min(i1, seqRows(rows, b, L));
  if (e <= i0) return;
  const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
  if (first >= L) {
    for (int i = i0; i < e; ++i) std::memset(MEM + off(ctx, (b * L + i) * hd + h * D), 0, size_t(D) << 2);
    return;
  }
  const int nk = last - first + 1;
  const bool dense = window == 0 && allKeys(off(mask, b * L), first, last);
  const uint32_t kp = off(scratch, L * L);
  packPanels(off(qkv, (b * L + first) * 3 * hd + (H + h) * D), 3 * hd, nk, D, kp);
  gemmP(off(qkv, (b * L + i0) * 3 * hd + h * D), 3 * hd, kp, scratch, L, e - i0, nk, D);
  for (int i = i0; i < e; ++i) {
    softmaxRow(off(scratch, (i - i0) * L), nk, off(mask, b * L), first, i, window, ldf(mask, b * L + i) > 0.5f,
               dense, scale);
  }
  gemmNN(scratch, L, off(qkv, (b * L + first) * 3 * hd + (2 * H + h) * D), 3 * hd,
         off(ctx, (b * L + i0) * hd + h * D), hd, e - i0, D, nk);
}

// src/wasm/plan.ts:795-840
void attrelf(uint32_t qkv, uint32_t posKey, uint32_t posQuery, uint32_t relidx, uint32_t mask, uint32_t ctx,
             uint32_t kinfo, uint32_t scratch, int L, int H, int D, float scale, int rows, int b, int h) {
  const int hd = H * D;
  const int S = 2 * L;
  const uint32_t c2p = off(scratch, L * L);
  const uint32_t p2c = off(c2p, L * S);
  const int nq = seqRows(rows, b, L);
  if (nq <= 0) return;
  const int first = ldi(kinfo, 2 * b), last = ldi(kinfo, 2 * b + 1);
  if (first >= L) {
    for (int i = 0; i < nq; ++i) std::memset(MEM + off(ctx, (b * L + i) * hd + h * D), 0, size_t(D) << 2);
    return;
  }
  const int nk = last - first + 1;
  const int lo = ldi(relidx, first * L + last);
  const int np = ldi(relidx, last * L + first) - lo + 1;
  const uint32_t q = off(qkv, b * L * 3 * hd);
  const float inv = 1.0f / scale;
  const bool dense = allKeys(off(mask, b * L), first, last);
  const uint32_t kp = off(p2c, L * S);
  packPanels(off(q, first * 3 * hd + (H + h) * D), 3 * hd, nk, D, kp);
  gemmP(off(q, h * D), 3 * hd, kp, scratch, L, nq, nk, D);
  packPanels(off(posKey, lo * hd + h * D), hd, np, D, kp);
  gemmP(off(q, h * D), 3 * hd, kp, c2p, S, nq, np, D);
  packPanels(off(posQuery, lo * hd + h * D), hd, np, D, kp);
  gemmP(off(q, first * 3 * hd + (H + h) * D), 3 * hd, kp, p2c, S, nk, np, D);
  for (int i = 0; i < nq; ++i) {
    const uint32_t p = off(scratch, i * L);
    const bool qm = ldf(mask, b * L + i) > 0.5f;
    if (qm) {
      for (int j = first; j <= last; ++j) {
        const int m = ldi(relidx, i * L + j) - lo;
        stf(p, j - first, (ldf(p, j - first) + ldf(c2p, i * S + m) + ldf(p2c, (j - first) * S + m)) * inv);
      }
    }
    softmaxRow(p, nk, off(mask, b * L), first, i, 0, qm, dense, 1);
  }
  gemmNN(scratch, L, off(q, first * 3 * hd + (2 * H + h) * D), 3 * hd, off(ctx, b * L * hd + h * D), hd, nq, D, nk);
}

// ---- stream (src/wasm/plan.ts:844-940) ----

inline uint32_t opAt(uint32_t stream, int o) { return stream + (uint32_t(HEAD + o * OPW) << 2); }
inline uint32_t ap(uint32_t op, int i) { return uint32_t(ldi(op, i + 2)); }
inline int32_t ai(uint32_t op, int i) { return ldi(op, i + 2); }
inline float af(uint32_t op, int i) { return ldf(op, i + 2); }
inline int rowsOf(uint32_t op, int rows) { const int f = ldi(op, 1); return f >= 0 ? f : rows; }
inline uint32_t scratchOf(uint32_t stream, int tid) {
  return uint32_t(ldi(stream, 5)) + uint32_t(tid) * uint32_t(ldi(stream, 6));
}

void serial(uint32_t stream, uint32_t op, int n) {
  const int batch = ldi(stream, 2);
  const uint32_t kinfo = uint32_t(ldi(stream, 4));
  const uint32_t scratch = scratchOf(stream, 0);
  const int code = ldi(op, 0);
  if (code == GEMM_P || code == GEMM_NT) {
    const int N = ai(op, 4), K = ai(op, 5);
    const int m = std::min(n, ai(op, 7));
    if (code == GEMM_P) {
      gemmP(ap(op, 0), K, ap(op, 1), ap(op, 3), N, m, N, K);
      if (ap(op, 2) || ai(op, 6)) biasAct(ap(op, 3), N, ap(op, 2), m, N, ai(op, 6));
    } else {
      gemmNT(ap(op, 0), K, ap(op, 1), K, ap(op, 3), N, ap(op, 2), m, N, K, 1, ai(op, 6));
    }
  } else if (code == LN) {
    layernorm(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), ap(op, 4), ap(op, 5), ai(op, 6), ai(op, 7), af(op, 8), 0, n);
  } else if (code == EMBLN) {
    embln(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), ap(op, 4), ap(op, 5), ap(op, 6), ap(op, 7), ai(op, 8),
          ai(op, 9), ai(op, 10), ai(op, 11), af(op, 12), ai(op, 13), ai(op, 14), n);
  } else if (code == ADD) {
    add(ap(op, 0), ap(op, 1), std::min(ai(op, 2), n * ai(op, 3)), ai(op, 3), ai(op, 4), ai(op, 5));
  } else if (code == GATHER) {
    gather(ap(op, 0), ap(op, 1), ap(op, 2), ai(op, 3), ai(op, 4), ai(op, 5), ai(op, 6));
  } else if (code == POOL) {
    pool(ap(op, 0), ap(op, 1), ap(op, 2), ai(op, 3), ai(op, 4), ai(op, 5), ai(op, 6));
  } else if (code == GEGLU) {
    geglu(ap(op, 0), ap(op, 1), ai(op, 2), 0, n);
  } else if (code == ROPE) {
    rope(ap(op, 0), ap(op, 1), ai(op, 2), ai(op, 3), ai(op, 4), n);
  } else if (code == IM2COL) {
    im2col(ap(op, 0), ap(op, 1), ap(op, 2), ai(op, 3), ai(op, 4), ai(op, 5), n);
  } else if (code == ATTSCORE) {
    attscore(ap(op, 0), ap(op, 1), kinfo, ai(op, 2), ai(op, 3), ai(op, 4), af(op, 5), n, batch);
  } else if (code == ATTSOFTMAX) {
    attsoftmax(ap(op, 0), ap(op, 1), kinfo, ai(op, 2), ai(op, 3), ai(op, 4), n);
  } else if (code == ATTPV) {
    attpv(ap(op, 0), ap(op, 1), ap(op, 2), kinfo, ai(op, 3), ai(op, 4), ai(op, 5), n, batch);
  } else if (code == ATTREL) {
    attrel(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), kinfo, ai(op, 4), ai(op, 5), ai(op, 6), ai(op, 7), ai(op, 8),
           ai(op, 9), n, batch);
  } else if (code == ATTSOFTREL) {
    attsoftrel(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), ap(op, 4), kinfo, ai(op, 5), ai(op, 6), ai(op, 7),
               ai(op, 8), af(op, 9), n);
  } else if (code == ATTSTD) {
    const int Lo = ai(op, 3);
    for (int b = 0; b < batch; ++b)
      for (int h = 0; h < ai(op, 4); ++h)
        attstdBlock(ap(op, 0), ap(op, 1), ap(op, 2), kinfo, scratch, Lo, ai(op, 4), ai(op, 5), af(op, 6), ai(op, 7),
                    n, b, h, 0, Lo);
  } else if (code == ATTRELF) {
    for (int b = 0; b < batch; ++b)
      for (int h = 0; h < ai(op, 7); ++h)
        attrelf(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), ap(op, 4), ap(op, 5), kinfo, scratch, ai(op, 6),
                ai(op, 7), ai(op, 8), af(op, 9), n, b, h);
  } else if (code == MASKLOGITS) {
    masklogits(ap(op, 0), ap(op, 1), ap(op, 2), ai(op, 3), af(op, 4), ai(op, 5));
  }
}

// ---- threads (src/wasm/plan.ts:942-1049) ----

struct Split { int rb, cb, qb, minWork; };
inline int cdiv(int a, int b) { return (a + b - 1) / b; }

int itemsOf(uint32_t stream, const Split& s, uint32_t op, int n) {
  const int code = ldi(op, 0);
  if (code == GEMM_P) {
    const int m = std::min(n, ai(op, 7));
    const int N = ai(op, 4);
    if (int64_t(m) * int64_t(N) * int64_t(ai(op, 5)) < int64_t(s.minWork)) return 0;
    return cdiv(m, s.rb) * cdiv(N, s.cb);
  }
  if (code == LN) return n >= 64 ? cdiv(n, 16) : 0;
  if (code == GEGLU) return n >= 16 ? cdiv(n, 8) : 0;
  if (code == ATTSTD) {
    const int batch = ldi(stream, 2);
    const int L = ai(op, 3);
    return batch * ai(op, 4) * cdiv(batch == 1 ? std::min(n, L) : L, s.qb);
  }
  if (code == ATTRELF) return ldi(stream, 2) * ai(op, 7);
  return 0;
}

void work(uint32_t stream, const Split& s, uint32_t op, int n, int i, int tid) {
  const int code = ldi(op, 0);
  if (code == GEMM_P) {
    const int N = ai(op, 4), K = ai(op, 5);
    const int m = std::min(n, ai(op, 7));
    const int nc = cdiv(N, s.cb);
    const int r0 = (i / nc) * s.rb, c0 = (i % nc) * s.cb;
    const int rr = std::min(s.rb, m - r0), cc = std::min(s.cb, N - c0);
    const uint32_t c = ap(op, 3) + (uint32_t(r0 * N + c0) << 2);
    gemmP(ap(op, 0) + (uint32_t(r0 * K) << 2), K, ap(op, 1) + uint32_t(c0 >> 4) * (uint32_t(K) << 6), c, N, rr, cc, K);
    const uint32_t bias = ap(op, 2);
    if (bias || ai(op, 6)) biasAct(c, N, bias ? bias + (uint32_t(c0) << 2) : 0, rr, cc, ai(op, 6));
  } else if (code == LN) {
    layernorm(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), ap(op, 4), ap(op, 5), ai(op, 6), ai(op, 7), af(op, 8),
              i * 16, std::min(n, i * 16 + 16));
  } else if (code == GEGLU) {
    geglu(ap(op, 0), ap(op, 1), ai(op, 2), i * 8, std::min(n, i * 8 + 8));
  } else if (code == ATTSTD) {
    const int batch = ldi(stream, 2);
    const int L = ai(op, 3), H = ai(op, 4);
    const int nb = cdiv(batch == 1 ? std::min(n, L) : L, s.qb);
    const int b = i / (H * nb), h = (i / nb) % H, q0 = (i % nb) * s.qb;
    attstdBlock(ap(op, 0), ap(op, 1), ap(op, 2), uint32_t(ldi(stream, 4)), scratchOf(stream, tid), L, H, ai(op, 5),
                af(op, 6), ai(op, 7), n, b, h, q0, q0 + s.qb);
  } else if (code == ATTRELF) {
    const int H = ai(op, 7);
    attrelf(ap(op, 0), ap(op, 1), ap(op, 2), ap(op, 3), ap(op, 4), ap(op, 5), uint32_t(ldi(stream, 4)),
            scratchOf(stream, tid), ai(op, 6), H, ai(op, 8), af(op, 9), n, i / H, i % H);
  }
}

// Helper pool: the coordinator publishes an op, helpers and the coordinator claim items from
// one atomic counter (src/wasm/plan.ts:1023-1049), the coordinator waits for every helper.
struct Pool {
  std::vector<std::thread> threads;
  std::mutex mu;
  std::condition_variable cv, done_cv;
  uint64_t gen = 0;
  bool stop = false;
  int pending = 0;
  std::atomic<int> next{0};
  uint32_t stream = 0, op = 0;
  int rows = 0, items = 0;
  Split split{16, 64, 32, 1 << 16};
  int nthreads = 1;

  void start(int n) {
    nthreads = n;
    for (int tid = 1; tid < n; ++tid) threads.emplace_back([this, tid] { helper(tid); });
  }
  void helper(int tid) {
    uint64_t seen = 0;
    for (;;) {
      uint32_t s_stream, s_op;
      int s_rows, s_items;
      {
        std::unique_lock<std::mutex> lk(mu);
        cv.wait(lk, [&] { return stop || gen != seen; });
        if (stop) return;
        seen = gen;
        s_stream = stream; s_op = op; s_rows = rows; s_items = items;
      }
      claim(s_stream, s_op, s_rows, s_items, tid);
      {
        std::lock_guard<std::mutex> lk(mu);
        if (--pending == 0) done_cv.notify_all();
      }
    }
  }
  void claim(uint32_t s_stream, uint32_t s_op, int s_rows, int s_items, int tid) {
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= s_items) break;
      work(s_stream, split, s_op, s_rows, i, tid);
    }
  }
  void parallel(uint32_t s_stream, uint32_t s_op, int n, int s_items) {
    {
      std::lock_guard<std::mutex> lk(mu);
      stream = s_stream; op = s_op; rows = n; items = s_items;
      next.store(0);
      pending = nthreads - 1;
      ++gen;
    }
    cv.notify_all();
    claim(s_stream, s_op, n, s_items, 0);
    std::unique_lock<std::mutex> lk(mu);
    done_cv.wait(lk, [&] { return pending == 0; });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
    }
    cv.notify_all();
    for (auto& t : threads) t.join();
  }
};

}  // namespace

extern "C" {

// Runs ops from .. to-1 of the stream at byte offset `stream` of `mem` over `rows` rows
// (src/wasm/plan.ts:855-873); the key ranges come from the mask at op 0. `pool` is a handle of
// oracle_threads_create or null for the serial executor.
void oracle_run_range(uint8_t* mem, uint32_t stream, int rows, int from, int to, void* pool) {
  MEM = mem;
  if (from == 0) keyRanges(uint32_t(ldi(stream, 3)), uint32_t(ldi(stream, 4)), ldi(stream, 1), ldi(stream, 2));
  Pool* p = static_cast<Pool*>(pool);
  for (int o = from; o < to; ++o) {
    const uint32_t op = opAt(stream, o);
    const int n = rowsOf(op, rows);
    const int items = (p && p->nthreads > 1) ? itemsOf(stream, p->split, op, n) : 0;
    if (items > 1) p->parallel(stream, op, n, items);
    else serial(stream, op, n);
  }
}

void oracle_run(uint8_t* mem, uint32_t stream, int rows, void* pool) {
  MEM = mem;
  oracle_run_range(mem, stream, rows, 0, ldi(stream, 0), pool);
}

// A helper pool of n threads (n - 1 helpers plus the caller) with the work split of
// src/plan/wasm.ts:123-124 (rb 16, cb 64, qb 32, minWork 65536) unless given.
void* oracle_threads_create(int n, int rb, int cb, int qb, int min_work) {
  Pool* p = new Pool();
  p->split = Split{rb, cb, qb, min_work};
  p->start(n < 1 ? 1 : n);
  return p;
}

void oracle_threads_destroy(void* pool) { delete static_cast<Pool*>(pool); }

// Scalar helpers exposed for the known-answer tests.
float oracle_vexp1(float x) { return vexp1(x); }
float oracle_vgelu1(float x) { return vgelu1(x); }
float oracle_gelu(float x) { return gelu(x); }

}  // extern "C"
