// CPU oracle for the wavo-b200 attention path.
//
// TEST INFRASTRUCTURE ONLY. This file restates, in C++, the reference's own CPU implementation of
// the attention path (vladkens/wavo, Rust: src/cpu/ops.rs, src/cpu/gemm.rs, src/cpu/mod.rs) so that
// the CUDA kernels can be checked against it and so that the reference CPU path can be timed on the
// host cores. Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and its
// `--impl reference` arm) may load it. No product code path calls into it.
//
// The reference is Rust and no Rust toolchain exists on this machine, so the reference itself cannot
// be built; this restatement follows it function by function (file:line cited at each function).
// Floating-point evaluation follows the reference exactly where the reference pins it: fused
// multiply-adds only where the reference uses `_mm256_fmadd_ps` / `mul_add`, every other operation
// separately rounded (the file is compiled with -ffp-contract=off).
//
// Parity pins: see tests/test_oracle.py. The oracle is checked against the naive references and the
// inputs of the reference's own unit tests (src/gpu/mod.rs:1717-2330, src/cpu/gemm.rs:567-657).

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <thread>
#include <vector>

#if !defined(__AVX2__) || !defined(__FMA__)
#error "the oracle is built for x86-64-v3 (AVX2 + FMA): see oracle/Makefile"
#endif

namespace {

// ---------------------------------------------------------------------------------------------
// Threads: src/cpu/mod.rs:79-111 (`threads`, `par_each`). Each call spawns its threads, which take
// the next item as they come free.
// ---------------------------------------------------------------------------------------------

int g_threads = 0;

int threads() {
  if (g_threads > 0) return g_threads;
  unsigned n = std::thread::hardware_concurrency();
  return n ? int(n) : 1;
}

void par_each(size_t items, const std::function<void(size_t)> &f) {
  size_t spawn = std::min<size_t>(size_t(threads()), items);
  if (spawn <= 1) {
    for (size_t i = 0; i < items; ++i) f(i);
    return;
  }
  std::atomic<size_t> next{0};
  auto work = [&]() {
    for (size_t i = next.fetch_add(1); i < items; i = next.fetch_add(1)) f(i);
  };
  std::vector<std::thread> pool;
  for (size_t t = 1; t < spawn; ++t) pool.emplace_back(work);
  work();
  for (auto &t : pool) t.join();
}

// ---------------------------------------------------------------------------------------------
// Scalars
// ---------------------------------------------------------------------------------------------

inline float from_bits(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}
inline uint32_t to_bits(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return b;
}

// src/cpu/gemm.rs:210-221 `to_half`: x rounded to the nearest f16 value (ties to even), kept as an
// f32; subnormal halves are multiples of 2^-24 and values past the f16 range keep their exponent.
inline float to_half(float x) {
  uint32_t b = to_bits(x);
  float normal = from_bits((b + 0xfffu + ((b >> 13) & 1u)) & 0xffffe000u);
  if (std::fabs(x) < from_bits(0x38800000u)) return std::nearbyint(x * 16777216.0f) / 16777216.0f;
  return normal;
}

// IEEE binary16 from f32, round to nearest even, overflow to infinity, NaN kept quiet: the
// conversion `half::f16::from_f32` (half 2.7.1) performs, as called at src/cpu/ops.rs:317 and
// src/cpu/transformer.rs (Decoder::pack). Written from the IEEE 754 definition.
inline uint16_t f16_bits(float x) {
  uint32_t b = to_bits(x);
  uint32_t sign = (b >> 16) & 0x8000u;
  uint32_t exp = (b >> 23) & 0xffu;
  uint32_t man = b & 0x7fffffu;
  if (exp == 0xffu) return uint16_t(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0u));
  int e = int(exp) - 127 + 15;
  if (e >= 0x1f) return uint16_t(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return uint16_t(sign);
    uint32_t m = man | 0x800000u;
    int shift = 14 - e;  // 24-bit significand down to the subnormal's 10 bits
    uint32_t half = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) half += 1;
    return uint16_t(sign | half);
  }
  uint32_t half = (uint32_t(e) << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half += 1;  // may carry into the exponent
  return uint16_t(sign | half);
}

inline float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (!man) return from_bits(sign);
    float v = float(man) * from_bits(0x33800000u);  // man * 2^-24, exact
    return sign ? -v : v;
  }
  if (exp == 0x1f) return from_bits(sign | 0x7f800000u | (man << 13));
  return from_bits(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

inline float f16_round(float x) { return f16_to_f32(f16_bits(x)); }

// src/cpu/ops.rs:12-26 `exp`: Cephes' expf without branches. Every operation rounds separately.
inline float cephes_exp(float x) {
  const float MAGIC = 12582912.0f;
  x = std::min(std::max(x, -87.0f), 88.0f);
  float t = x * 1.44269504088896340736f + MAGIC;
  float n = t - MAGIC;
  float r = x - n * 0.6933594f + n * 2.1219444e-4f;
  float p = 1.9875691e-4f * r + 1.3981999e-3f;
  p = ((((p * r + 8.333452e-3f) * r + 4.1665796e-2f) * r + 0.16666665f) * r + 0.5f) * r * r;
  uint32_t bits = (uint32_t(int32_t(to_bits(t)) - 0x4B400000 + 127)) << 23;
  return (p + r + 1.0f) * from_bits(bits);
}

// src/cpu/ops.rs:28-40
inline float silu(float x) { return x / (1.0f + cephes_exp(-x)); }
inline float signum(float x) { return std::signbit(x) ? -1.0f : 1.0f; }
inline float gelu(float x) {
  float z = std::fabs(0.70710678118654752440f * x);
  float t = 1.0f / (1.0f + 0.3275911f * z);
  float p = (((1.0614054f * t - 1.453152f) * t + 1.4214138f) * t - 0.28449674f) * t + 0.2548296f;
  return 0.5f * x * (1.0f + signum(x) * (1.0f - p * t * cephes_exp(-z * z)));
}

// src/cpu/ops.rs:55-63 `sum`: 8 lanes, then the lanes in order.
inline float sum8(const float *v, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t i = 0; i < n; ++i) acc[i % 8] += v[i];
  float s = 0.0f;
  for (int i = 0; i < 8; ++i) s += acc[i];
  return s;
}

// src/cpu/mod.rs:356-380 (x86 `sum` and `dot`): two 8-float FMA accumulators over chunks of 16,
// the pairwise reduction of `sum`, then the tail in order.
inline float hsum16(__m256 a, __m256 b) {
  __m256 s = _mm256_add_ps(a, b);
  __m128 q = _mm_add_ps(_mm256_castps256_ps128(s), _mm256_extractf128_ps(s, 1));
  q = _mm_add_ps(q, _mm_movehl_ps(q, q));
  return _mm_cvtss_f32(q) + _mm_cvtss_f32(_mm_shuffle_ps(q, q, 1));
}

float dot(const float *a, const float *b, size_t len) {
  size_t n = len / 16 * 16;
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  for (size_t i = 0; i < n; i += 16) {
    acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc0);
    acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), acc1);
  }
  float tail = 0.0f;
  for (size_t i = n; i < len; ++i) tail += a[i] * b[i];
  return hsum16(acc0, acc1) + tail;
}

// ---------------------------------------------------------------------------------------------
// Panels and tiles: src/cpu/gemm.rs:23-28, 271-302, 354-377, 502-529
// ---------------------------------------------------------------------------------------------

constexpr size_t NR = 16;  // panel width
constexpr size_t MR = 6;   // rows of `a` per tile

inline size_t ceil_to(size_t x, size_t m) { return (x + m - 1) / m * m; }

// src/cpu/gemm.rs:271-285 `panels`: the panels [k][NR] of b (a matrix [n][k] with row stride ld, or
// with `transposed` [k][n]); zeros past n and past `rows` rows up to k.
std::vector<float> panels(const float *b, size_t ld, size_t n, size_t k, size_t rows,
                          bool transposed) {
  std::vector<float> out((n + NR - 1) / NR * k * NR, 0.0f);
  for (size_t p = 0; p * NR < n; ++p) {
    float *o = out.data() + p * k * NR;
    for (size_t j = 0; j < std::min(NR, n - NR * p); ++j) {
      size_t col = NR * p + j;
      for (size_t kk = 0; kk < rows; ++kk)
        o[kk * NR + j] = transposed ? b[kk * ld + col] : b[col * ld + kk];
    }
  }
  return out;
}

// src/cpu/gemm.rs:502-529 (x86 `tile`): MR rows of a times a panel [k][NR]; per output one FMA
// chain over k in order.
inline void tile(const float *const a[MR], const float *b, size_t k, float out[MR][NR]) {
  __m256 acc[MR][2];
  for (size_t r = 0; r < MR; ++r) acc[r][0] = acc[r][1] = _mm256_setzero_ps();
  for (size_t kk = 0; kk < k; ++kk) {
    __m256 b0 = _mm256_loadu_ps(b + kk * NR), b1 = _mm256_loadu_ps(b + kk * NR + 8);
    for (size_t r = 0; r < MR; ++r) {
      __m256 v = _mm256_broadcast_ss(a[r] + kk);
      acc[r][0] = _mm256_fmadd_ps(v, b0, acc[r][0]);
      acc[r][1] = _mm256_fmadd_ps(v, b1, acc[r][1]);
    }
  }
  for (size_t r = 0; r < MR; ++r) {
    _mm256_storeu_ps(out[r], acc[r][0]);
    _mm256_storeu_ps(out[r] + 8, acc[r][1]);
  }
}

// src/cpu/gemm.rs:287-302 `product`: c = a·b for m rows of a (stride lda, k long), b as panels;
// all the panels' columns of c (stride ldc). The store adds a zero bias (`finish` with ZEROS).
void product(const float *a, size_t lda, size_t m, const float *b, size_t b_len, size_t k,
             float *c, size_t ldc) {
  size_t np = b_len / (k * NR);
  float acc[MR][NR];
  for (size_t i = 0; i < m; i += MR) {
    const float *rows[MR];
    for (size_t r = 0; r < MR; ++r) rows[r] = a + std::min(i + r, m - 1) * lda;
    for (size_t p = 0; p < np; ++p) {
      tile(rows, b + p * k * NR, k, acc);
      for (size_t r = 0; r < MR && i + r < m; ++r)
        for (size_t j = 0; j < NR; ++j) c[(i + r) * ldc + NR * p + j] = acc[r][j] + 0.0f;
    }
  }
}

// src/cpu/ops.rs:275-287 `softmax`: scores × scale over the first t of each of m rows (rows of
// ceil16(t)); the rest of each row zeroed.
void softmax(float *scores, size_t m, size_t t, float scale) {
  size_t tp = ceil_to(t, NR);
  for (size_t r = 0; r < m; ++r) {
    float *row = scores + r * tp;
    float mx = -INFINITY;
    for (size_t j = 0; j < t; ++j) mx = std::fmax(mx, row[j]);
    mx = mx * scale;
    for (size_t j = 0; j < t; ++j) row[j] = cephes_exp(row[j] * scale - mx);
    float inv = 1.0f / sum8(row, t);
    for (size_t j = 0; j < t; ++j) row[j] *= inv;
    for (size_t j = t; j < tp; ++j) row[j] = 0.0f;
  }
}

constexpr size_t QUERIES = 48;  // src/cpu/ops.rs:184-185

}  // namespace

// =============================================================================================
// C ABI (ctypes)
// =============================================================================================

extern "C" {

void wo_set_threads(int n) { g_threads = n; }
int wo_threads(void) { return threads(); }

// src/gpu/mod.rs:1717-1727 (the reference tests' `random`): xorshift32, values in [-1, 1].
void wo_random(float *out, size_t n, uint32_t seed) {
  uint32_t x = (seed * 2654435761u) | 1u;
  const float max = float(UINT32_MAX);
  for (size_t i = 0; i < n; ++i) {
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    out[i] = float(x) / max * 2.0f - 1.0f;
  }
}

float wo_to_half(float x) { return to_half(x); }
void wo_to_half_n(const float *x, float *y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = to_half(x[i]);
}
uint16_t wo_f16_bits(float x) { return f16_bits(x); }
float wo_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
void wo_f16_round_n(const float *x, float *y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = f16_round(x[i]);
}
float wo_exp(float x) { return cephes_exp(x); }
float wo_silu(float x) { return silu(x); }
float wo_gelu(float x) { return gelu(x); }
float wo_dot(const float *a, const float *b, size_t n) { return dot(a, b, n); }

// src/cpu/ops.rs:187-221 `attention`: row i's q at qk[i·ld..], its k at qk[i·ld + ch..], its v at
// v[i·ldv..], into o [t][ch]; one head per job, 48 queries per step.
void wo_attention(const float *qk, size_t ld, const float *v, size_t ldv, float *o, size_t t,
                  size_t heads, size_t ch) {
  size_t hd = ch / heads, tp = ceil_to(t, NR), hp = ceil_to(hd, NR);
  float scale = 1.0f / std::sqrt(float(hd));
  std::vector<std::vector<float>> outs(heads);
  par_each(heads, [&](size_t h) {
    std::vector<float> s(QUERIES * tp);
    std::vector<float> keys = panels(qk + ch + h * hd, ld, t, hd, hd, false);
    std::vector<float> values = panels(v + h * hd, ldv, hd, tp, t, true);
    std::vector<float> &out = outs[h];
    out.assign(t * hp, 0.0f);
    for (size_t i = 0; i < t; i += QUERIES) {
      size_t m = std::min(QUERIES, t - i);
      product(qk + i * ld + h * hd, ld, m, keys.data(), keys.size(), hd, s.data(), tp);
      softmax(s.data(), m, t, scale);
      product(s.data(), tp, m, values.data(), values.size(), tp, out.data() + i * hp, hp);
    }
  });
  // src/cpu/ops.rs:289-298 `gather`
  for (size_t h = 0; h < heads; ++h)
    for (size_t r = 0; r < t; ++r) std::memcpy(o + r * ch + h * hd, outs[h].data() + r * hp, hd * 4);
}

// src/gpu/mod.rs:1060-1065 `pos_rows`
size_t wo_pos_rows(size_t t) { return 2 * t + 15; }

// src/cpu/ops.rs:223-273 `relative_attention`: qkv [t][q | k | v], pos the projected positions
// [pos_rows(t)][ch] (row r is position t + 15 - r), u and v [heads][hd]; score (i, j) is
// ((q + u)_i·k_j + (q + v)_i·pos[j - i + t + 15]) / sqrt(hd). Heads of a multiple of 16 dims, as
// the reference asserts (its `product` needs the value panels to fit the output rows); returns -1
// otherwise.
int wo_relative_attention(const float *qkv, const float *pos, const float *u, const float *vb,
                          float *o, size_t t, size_t heads, size_t ch) {
  size_t hd = ch / heads, tp = ceil_to(t, NR);
  if (hd % NR != 0) return -1;
  size_t pw = ceil_to(t + QUERIES + 2 * NR, NR);
  float scale = 1.0f / std::sqrt(float(hd));
  std::vector<std::vector<float>> outs(heads);
  par_each(heads, [&](size_t h) {
    std::vector<float> s(QUERIES * tp), sp(QUERIES * pw);
    std::vector<float> keys = panels(qkv + ch + h * hd, 3 * ch, t, hd, hd, false);
    std::vector<float> values = panels(qkv + 2 * ch + h * hd, 3 * ch, hd, tp, t, true);
    std::vector<float> positions = panels(pos + h * hd, ch, 2 * t + 15, hd, hd, false);
    std::vector<float> qu(t * hd), qv(t * hd);
    for (size_t r = 0; r < t; ++r)
      for (size_t c = 0; c < hd; ++c) {
        float q = qkv[r * 3 * ch + h * hd + c];
        qu[r * hd + c] = q + u[h * hd + c];
        qv[r * hd + c] = q + vb[h * hd + c];
      }
    std::vector<float> &out = outs[h];
    out.assign(t * hd, 0.0f);
    for (size_t i = 0; i < t; i += QUERIES) {
      size_t m = std::min(QUERIES, t - i);
      product(qu.data() + i * hd, hd, m, keys.data(), keys.size(), hd, s.data(), tp);
      size_t p0 = (t + 16 - i - m) / NR, p1 = (2 * t + 15 - i + NR - 1) / NR;
      product(qv.data() + i * hd, hd, m, positions.data() + p0 * NR * hd, (p1 - p0) * NR * hd, hd,
              sp.data(), pw);
      for (size_t a = 0; a < m; ++a) {
        // Query i + a, key j: position row j - i - a + t + 15, from p0·NR on.
        const float *row = sp.data() + a * pw + (t + 15 - i - a - p0 * NR);
        float *srow = s.data() + a * tp;
        for (size_t j = 0; j < t; ++j) srow[j] += row[j];
      }
      softmax(s.data(), m, t, scale);
      product(s.data(), tp, m, values.data(), values.size(), tp, out.data() + i * hd, hd);
    }
  });
  for (size_t h = 0; h < heads; ++h)
    for (size_t r = 0; r < t; ++r) std::memcpy(o + r * ch + h * hd, outs[h].data() + r * hd, hd * 4);
  return 0;
}

// src/cpu/ops.rs:300-337 `attend`: one query per head, q [heads][hd] rounded to f16, over the first
// n positions of a cache kv (K, then V, each [heads][cols][hd]), into o [heads][hd].
void wo_attend(const float *q, const float *kv, size_t cols, size_t n, float *o, size_t heads,
               size_t hd) {
  float scale = 1.0f / std::sqrt(float(hd));
  const float *k = kv, *v = kv + heads * cols * hd;
  size_t jobs = std::min(std::max<size_t>((heads * n * hd) >> 16, 1), heads);
  size_t per = (heads + jobs - 1) / jobs;
  size_t njobs = (heads + per - 1) / per;
  par_each(njobs, [&](size_t jb) {
    std::vector<float> qh(hd), s(n);
    for (size_t h = jb * per; h < std::min(heads, (jb + 1) * per); ++h) {
      for (size_t c = 0; c < hd; ++c) qh[c] = f16_round(q[h * hd + c]);
      const float *kh = k + h * cols * hd, *vh = v + h * cols * hd;
      for (size_t j = 0; j < n; ++j) s[j] = dot(qh.data(), kh + j * hd, hd) * scale;
      float mx = -INFINITY;
      for (size_t j = 0; j < n; ++j) mx = std::fmax(mx, s[j]);
      for (size_t j = 0; j < n; ++j) s[j] = cephes_exp(s[j] - mx);
      float inv = 1.0f / sum8(s.data(), n);
      float *oh = o + h * hd;
      for (size_t c = 0; c < hd; ++c) oh[c] = 0.0f;
      for (size_t j = 0; j < n; ++j)
        for (size_t c = 0; c < hd; ++c) oh[c] += s[j] * vh[j * hd + c];
      for (size_t c = 0; c < hd; ++c) oh[c] *= inv;
    }
  });
}

// src/cpu/transformer.rs:209-222 `Decoder::pack`: rows [k | v] of kv (2·d floats each) into the
// cache (K heads then V heads, each [cols][hd]) at positions col.., rounded to f16.
void wo_pack_cache(const float *kv, size_t rows, size_t d, size_t hd, float *cache, size_t cols,
                   size_t col) {
  for (size_t j = 0; j < rows; ++j)
    for (size_t h = 0; h < 2 * d / hd; ++h) {
      size_t at = (h * cols + col + j) * hd;
      for (size_t c = 0; c < hd; ++c) cache[at + c] = f16_round(kv[j * 2 * d + h * hd + c]);
    }
}

// src/cpu/ops.rs:339-355 `rope`: in place over rows [q | k | v] of heads × hd, row j at table row
// j (rot/2 cosines then rot/2 sines); pairs (2i, 2i+1), or with neox (i, i + rot/2), of q's and k's
// heads rotate.
void wo_rope(float *qkv, const float *table, size_t rows, size_t heads, size_t hd, size_t rot,
             int neox) {
  size_t half = rot / 2, pair = neox ? half : 1, step = neox ? 1 : 2;
  for (size_t r = 0; r < rows; ++r) {
    float *row = qkv + r * 3 * heads * hd;
    const float *cs = table + r * rot, *sn = cs + half;
    for (size_t hh = 0; hh < 2 * heads; ++hh) {
      float *head = row + hh * hd;
      for (size_t i = 0; i < half; ++i) {
        float a = head[step * i], b = head[step * i + pair];
        head[step * i] = a * cs[i] - b * sn[i];
        head[step * i + pair] = a * sn[i] + b * cs[i];
      }
    }
  }
}

// src/cpu/ops.rs:47-53 `moments`: mean and 1/sqrt(variance + 1e-5) of a row, both sums by `sum`.
static void moments(const float *x, size_t n, float &mean, float &rstd) {
  const float fn = float(n);
  mean = sum8(x, n) / fn;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t i = 0; i < n; ++i) {
    const float d = x[i] - mean;
    acc[i % 8] += d * d;
  }
  float var = 0.0f;
  for (int i = 0; i < 8; ++i) var += acc[i];
  var /= fn;
  rstd = 1.0f / std::sqrt(var + 1e-5f);
}

// src/cpu/ops.rs:65-110 `layer_norm`: y = (x - mean)·rstd·w + b per row of `cols`; with a table
// (rows of hd / 2 cosines then as many sines, row r for row r) also yr = y with NEOX rotary pairs
// (i, i + hd/2) rotated inside each head of hd.
void wo_layer_norm(const float *x, const float *w, const float *b, float *y, size_t rows,
                   size_t cols, const float *table, float *yr, size_t hd) {
  par_each(rows, [&](size_t r) {
    const float *xr = x + r * cols;
    float *yy = y + r * cols;
    float mean, rstd;
    moments(xr, cols, mean, rstd);
    for (size_t c = 0; c < cols; ++c) yy[c] = (xr[c] - mean) * rstd * w[c] + b[c];
    if (!table) return;
    const size_t half = hd / 2;
    const float *cs = table + r * hd, *sn = cs + half;
    for (size_t h0 = 0; h0 + hd <= cols; h0 += hd) {
      const float *y0 = yy + h0, *y1 = yy + h0 + half;
      float *r0 = yr + r * cols + h0, *r1 = r0 + half;
      for (size_t i = 0; i < half; ++i) {
        r0[i] = y0[i] * cs[i] - y1[i] * sn[i];
        r1[i] = y1[i] * cs[i] + y0[i] * sn[i];
      }
    }
  });
}

// src/cpu/ops.rs:133-182 `conv_glu`: the Conformer conv module between the pointwise convs. GLU of
// h [t][2·ch] in place into its first halves (x /= 1 + exp(-gate)), the depthwise conv (odd
// kernel, centred, taps [kernel][ch] and bias) over frames of the segment, then LayerNorm over the
// channels (`moments`) or the per-channel affine (g, beta), SiLU, into y [t][ch].
void wo_conv_glu(float *h, const float *taps, const float *bias, const float *g, const float *beta,
                 int layer_norm, float *y, size_t t, size_t ch, size_t kernel) {
  par_each(t, [&](size_t i) {
    float *x = h + i * 2 * ch;
    const float *gate = x + ch;
    for (size_t c = 0; c < ch; ++c) x[c] /= 1.0f + cephes_exp(-gate[c]);
  });
  par_each(t, [&](size_t i) {
    std::vector<float> acc(bias, bias + ch);
    for (size_t k = 0; k < kernel; ++k) {
      if (i + k < kernel / 2) continue;
      const size_t src = i + k - kernel / 2;
      if (src >= t) continue;
      const float *tk = taps + k * ch, *xs = h + src * 2 * ch;
      for (size_t c = 0; c < ch; ++c) acc[c] += tk[c] * xs[c];
    }
    float mean = 0.0f, rstd = 1.0f;
    if (layer_norm) moments(acc.data(), ch, mean, rstd);
    float *yy = y + i * ch;
    for (size_t c = 0; c < ch; ++c) yy[c] = silu((acc[c] - mean) * rstd * g[c] + beta[c]);
  });
}

// src/whisper/search.rs:46-59 `pick` with `timestamp_rules` (76-107) and `argmax` (111-123): the
// suppression lists, the timestamp rules over the window's generated tokens, the first maximum and
// (with logprob) its log-softmax; logits edited in place. Returns the token.
int wo_pick(float *logits, size_t vocab, const int32_t *generated, size_t n,
            const int32_t *suppress, size_t n_suppress, const int32_t *begin_suppress,
            size_t n_begin, size_t eot, size_t no_ts, size_t begin, size_t max_initial,
            int logprob, float *lp_out) {
  const float ninf = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < n_suppress; ++i) logits[suppress[i]] = ninf;
  if (n == 0)
    for (size_t i = 0; i < n_begin; ++i) logits[begin_suppress[i]] = ninf;
  // timestamp_rules
  auto is_ts = [&](int32_t id) { return size_t(id) >= begin; };
  logits[no_ts] = ninf;
  const bool last = n > 0 && is_ts(generated[n - 1]);
  const bool penultimate = n < 2 || is_ts(generated[n - 2]);
  if (last) {
    const size_t lo = penultimate ? begin : 0, hi = penultimate ? vocab : eot;
    for (size_t i = lo; i < hi; ++i) logits[i] = ninf;
  }
  for (size_t i = n; i-- > 0;) {
    if (is_ts(generated[i])) {
      const size_t ts = size_t(generated[i]);
      const size_t low = (last && !penultimate) ? ts : ts + 1;
      for (size_t j = begin; j < low; ++j) logits[j] = ninf;
      break;
    }
  }
  if (n == 0) {
    for (size_t i = 0; i < begin; ++i) logits[i] = ninf;
    const size_t end = std::min(begin + max_initial + 1, vocab);
    for (size_t i = end; i < vocab; ++i) logits[i] = ninf;
  }
  float mx = ninf;
  for (size_t i = begin; i < vocab; ++i) mx = std::max(mx, logits[i]);
  float mass = ninf;
  if (std::isfinite(mx)) {
    double sum = 0.0;
    for (size_t i = begin; i < vocab; ++i)
      if (std::isfinite(logits[i])) sum += std::exp(double(logits[i] - mx));
    if (sum > 0.0) mass = mx + float(std::log(sum));
  }
  float text = ninf;
  for (size_t i = 0; i < begin; ++i) text = std::max(text, logits[i]);
  if (mass > text)
    for (size_t i = 0; i < begin; ++i) logits[i] = ninf;
  // argmax
  size_t best = 0;
  for (size_t i = 0; i < vocab; ++i)
    if (logits[i] > logits[best]) best = i;
  float lp = 0.0f;
  if (logprob) {
    float m = ninf;
    for (size_t i = 0; i < vocab; ++i)
      if (std::isfinite(logits[i])) m = std::max(m, logits[i]);
    double sum = 0.0;
    for (size_t i = 0; i < vocab; ++i)
      if (std::isfinite(logits[i])) sum += std::exp(double(logits[i] - m));
    lp = logits[best] - (m + float(std::log(sum)));
  }
  if (lp_out) *lp_out = lp;
  return int(best);
}

// src/gigaam/mod.rs:88-96 `rope`: per position hd/2 cosines then hd/2 sines, angles in f64.
void wo_rope_table(size_t frames, size_t hd, double theta, float *out) {
  for (size_t t = 0; t < frames; ++t)
    for (size_t i = 0; i < hd / 2; ++i) {
      double a = double(t) * std::pow(theta, -2.0 * double(i) / double(hd));
      out[t * hd + i] = float(std::cos(a));
      out[t * hd + hd / 2 + i] = float(std::sin(a));
    }
}

// src/conformer.rs:141-153 `rel_positions`: the sinusoidal table of positions first, first - 1, …
// for rows rows of d: [2k] = sin(pos·d_k), [2k + 1] = cos(pos·d_k), in f32.
void wo_rel_positions(size_t d, int64_t first, size_t rows, float *out) {
  std::vector<float> div(d / 2);
  float c = -std::log(10000.0f) / float(d);
  for (size_t k = 0; k < d / 2; ++k) div[k] = std::exp(float(2 * k) * c);
  for (size_t r = 0; r < rows; ++r) {
    float p = float(first - int64_t(r));
    for (size_t k = 0; k < d / 2; ++k) {
      out[r * d + 2 * k] = std::sin(p * div[k]);
      out[r * d + 2 * k + 1] = std::cos(p * div[k]);
    }
  }
}

}  // extern "C"

// =============================================================================================
// Linear layers and the projection GEMM: src/cpu/gemm.rs:30-177, src/cpu/mod.rs:237-261
// =============================================================================================

namespace {

enum Ty { TY_F32 = 0, TY_F16 = 1, TY_Q8_0 = 8 };  // GGUF type ids, src/gguf.rs:14-38

enum Epi { E_BIAS = 0, E_SILU, E_RELU, E_RESIDUAL, E_GELU, E_GELU_RESIDUAL, E_TANH };

struct Linear {
  size_t n, k;
  int ty;
  std::vector<float> f32;      // F32
  std::vector<uint16_t> f16;   // F16 bits
  std::vector<int8_t> q;       // Q8_0 values [n][k]
  std::vector<float> d;        // Q8_0 scales [n][k/32]
  std::vector<float> bias;     // n values
};

// src/cpu/gemm.rs:339-352 `finish`
inline void finish(float *c, const float *acc, const float *bias, size_t len, int epi,
                   float alpha) {
  for (size_t i = 0; i < len; ++i) {
    float v = acc[i] + bias[i];
    switch (epi) {
      case E_BIAS: c[i] = v; break;
      case E_SILU: c[i] = silu(v); break;
      case E_RELU: c[i] = std::fmax(v, 0.0f); break;
      case E_RESIDUAL: c[i] += alpha * v; break;
      case E_GELU: c[i] = gelu(v); break;
      case E_GELU_RESIDUAL: c[i] += gelu(v); break;
      default: c[i] = std::tanh(std::min(std::max(v, -10.0f), 10.0f)); break;
    }
  }
}

// src/cpu/gemm.rs:87-122 `Linear::pack`: panel p as f32 [k][NR], W rounded to f16 (F16 exact).
void pack_panel(const Linear &l, size_t p, float *out) {
  size_t k = l.k;
  for (size_t j = 0; j < NR; ++j) {
    size_t row = NR * p + j;
    for (size_t kk = 0; kk < k; ++kk) {
      float w = 0.0f;
      if (row < l.n) {
        if (l.ty == TY_Q8_0) w = to_half(float(l.q[row * k + kk]) * l.d[row * k / 32 + kk / 32]);
        else if (l.ty == TY_F16) w = f16_to_f32(l.f16[row * k + kk]);
        else w = to_half(l.f32[row * k + kk]);
      }
      out[kk * NR + j] = w;
    }
  }
}

// CPUID: AVX-VNNI (leaf 7.1 EAX bit 4) or AVX512-VNNI with AVX512VL (leaf 7.0 ECX bit 11, EBX bit 31).
// src/cpu/mod.rs:339-354 `vnni`.
int detect_vnni() {
  unsigned a, b, c, d;
  __asm__ volatile("cpuid" : "=a"(a), "=b"(b), "=c"(c), "=d"(d) : "a"(7), "c"(1));
  if (a & (1u << 4)) return 1;
  __asm__ volatile("cpuid" : "=a"(a), "=b"(b), "=c"(c), "=d"(d) : "a"(7), "c"(0));
  if ((c & (1u << 11)) && (b & (1u << 31))) return 2;
  return 0;
}
int g_vnni = -1;  // -1: detect; 0: off (the f16 path); 1/2: on

// src/cpu/gemm.rs:385-407 `x86::quantize`: rows per 32 values as i16 q and a scale d,
// q = round(x / d) (x · 32767 / max, rounded to nearest even, saturated), d = max|x| / 32767.
void quantize(const float *x, int16_t *q, float *d, size_t blocks) {
  for (size_t blk = 0; blk < blocks; ++blk) {
    const float *v = x + 32 * blk;
    float mx = 0.0f;
    for (int i = 0; i < 32; ++i) mx = std::fmax(mx, std::fabs(v[i]));
    d[blk] = mx / 32767.0f;
    float id = mx > 0.0f ? 32767.0f / mx : 0.0f;
    for (int i = 0; i < 32; ++i) {
      float s = v[i] * id;
      long r = std::lrintf(s);  // round to nearest even, as cvtps_epi32
      if (!(s == s) || s >= 2147483648.0f || s < -2147483648.0f) r = INT32_MIN;
      q[32 * blk + i] = int16_t(std::min<long>(std::max<long>(r, -32768), 32767));
    }
  }
}

}  // namespace

// ---- the log-mel frontend (src/parakeet/frontend.rs, src/fft.rs) -----------------------------

namespace {

constexpr double kTau = 6.283185307179586;

// src/fft.rs:40-143 `Fft<f64>`: radix-2 decimation in time down to naive DFTs of the odd factor,
// the data in Stockham order; every multiply-add fused as the reference's `mul_add`.
struct RealFft {
  size_t n = 0, leaf = 0, blocks = 0;
  std::vector<size_t> perm;
  std::vector<double> lcos, lsin;  // [j][k]
  std::vector<double> tcos, tsin;  // [stage][n / 2]
  explicit RealFft(size_t n_) : n(n_) {
    size_t tz = 0;
    while (((n >> tz) & 1) == 0) ++tz;
    leaf = n >> tz;
    blocks = n / leaf;
    std::vector<size_t> starts{0};
    while (starts.size() < blocks) {
      std::vector<size_t> next;
      for (size_t v : starts) next.push_back(2 * v);
      for (size_t v : starts) next.push_back(2 * v + 1);
      starts = next;
    }
    for (size_t i = 0; i < n; ++i) perm.push_back(starts[i % blocks] + i / blocks * blocks);
    auto trig = [&](size_t i, std::vector<double> &c, std::vector<double> &s) {
      const double phase = kTau * double(i) / double(n);
      c.push_back(std::cos(phase));
      s.push_back(std::sin(phase));
    };
    for (size_t i = 0; i < leaf * leaf; ++i) trig(i / leaf * (i % leaf) * blocks % n, lcos, lsin);
    for (size_t size = 2 * leaf; size <= n; size *= 2)
      for (size_t i = 0; i < n / 2; ++i) trig(i / (n / size) * (n / size), tcos, tsin);
  }
  // re and im of the n real values x (src/fft.rs:86-143 `run`, `leaves`, `stage`).
  void forward(const double *x, double *re, double *im) const {
    const size_t stages = tcos.size() / (n / 2);
    std::vector<double> buf(4 * n, 0.0);
    double *front = buf.data(), *back = buf.data() + 2 * n;
    double *src = stages % 2 == 0 ? back : front, *dst = stages % 2 == 0 ? front : back;
    for (size_t v = 0; v < n; ++v) src[v] = x[perm[v]];
    for (size_t k = 0; k < leaf; ++k) {
      double *r = dst + k * blocks, *m = dst + n + k * blocks;
      for (size_t g = 0; g < blocks; ++g) {
        r[g] = src[g];
        m[g] = 0.0;
      }
      for (size_t j = 1; j < leaf; ++j) {
        const double c = lcos[j * leaf + k], s = lsin[j * leaf + k];
        const double *xs = src + j * blocks;
        for (size_t g = 0; g < blocks; ++g) {
          r[g] = std::fma(xs[g], c, r[g]);
          m[g] = std::fma(-xs[g], s, m[g]);
        }
      }
    }
    const size_t half = n / 2;
    for (size_t st = 0; st < stages; ++st) {
      std::swap(src, dst);
      const double *sr = src, *si = src + n, *cs = tcos.data() + st * half, *sn = tsin.data() + st * half;
      double *dr = dst, *di = dst + n;
      for (size_t i = 0; i < half; ++i) {
        const double c = cs[i], s = sn[i], a = sr[2 * i], xv = sr[2 * i + 1], b = si[2 * i],
                     y = si[2 * i + 1];
        dr[i] = std::fma(s, y, std::fma(c, xv, a));
        di[i] = std::fma(-s, xv, std::fma(c, y, b));
        dr[i + half] = std::fma(-s, y, std::fma(-c, xv, a));
        di[i + half] = std::fma(s, xv, std::fma(-c, y, b));
      }
    }
    std::memcpy(re, dst, n * sizeof(double));
    std::memcpy(im, dst + n, n * sizeof(double));
  }
};

constexpr size_t kMels = 128, kNfft = 512, kWindow = 400, kHop = 160, kBins = kNfft / 2 + 1;
constexpr float kPreEmphasis = 0.97f, kFMax = 8000.0f;
const float kLogEps = 1.0f / float(1 << 24);

// src/parakeet/frontend.rs:110-140 `slaney_filterbank`: librosa's mel(16000, 512, 128, 0, 8000,
// norm='slaney') computed in f64, stored as f32.
std::vector<float> slaney_filterbank() {
  const double fsp = 200.0 / 3.0, min_log_hz = 1000.0;
  const double min_log_mel = min_log_hz / fsp, log_step = std::log(6.4) / 27.0;
  auto hz_to_mel = [&](double hz) {
    return hz < min_log_hz ? hz / fsp : min_log_mel + std::log(hz / min_log_hz) / log_step;
  };
  auto mel_to_hz = [&](double mel) {
    return mel < min_log_mel ? mel * fsp : min_log_hz * std::exp(log_step * (mel - min_log_mel));
  };
  const double mel_max = hz_to_mel(double(kFMax));
  std::vector<double> hz(kMels + 2);
  for (size_t m = 0; m < kMels + 2; ++m) hz[m] = mel_to_hz(mel_max * double(m) / double(kMels + 1));
  std::vector<float> out(kMels * kBins, 0.0f);
  for (size_t m = 0; m < kMels; ++m) {
    const double enorm = 2.0 / (hz[m + 2] - hz[m]);
    for (size_t k = 0; k < kBins; ++k) {
      const double f = 16000.0 * double(k) / double(kNfft);
      const double lower = (f - hz[m]) / (hz[m + 1] - hz[m]);
      const double upper = (hz[m + 2] - f) / (hz[m + 2] - hz[m + 1]);
      out[m * kBins + k] = float(std::max(std::min(lower, upper), 0.0) * enorm);
    }
  }
  return out;
}

struct Frontend {
  std::vector<double> window;
  std::vector<float> filters;
  std::vector<std::pair<size_t, size_t>> spans;
  RealFft fft{kNfft};
  Frontend() {
    const size_t pad = (kNfft - kWindow) / 2;
    for (size_t i = 0; i < kNfft; ++i) {
      const size_t k = i - pad;  // wraps below pad, as the reference's wrapping_sub
      window.push_back(k < kWindow ? 0.5 - 0.5 * std::cos(2.0 * M_PI * double(k) / double(kWindow - 1))
                                   : 0.0);
    }
    filters = slaney_filterbank();
    for (size_t m = 0; m < kMels; ++m) {
      const float *f = filters.data() + m * kBins;
      size_t lo = 0;
      while (lo < kBins && f[lo] == 0.0f) ++lo;
      if (lo == kBins) {
        spans.push_back({0, 0});
        continue;
      }
      size_t hi = kBins;
      while (hi > lo && f[hi - 1] == 0.0f) --hi;
      spans.push_back({lo, hi});
    }
  }
  // src/parakeet/frontend.rs:74-108 `log_mel`: frames [f0, f1) of the whole pcm, time-major.
  void log_mel(const float *pcm, size_t n_pcm, size_t f0, size_t f1, float *out) const {
    const size_t frames = f1 - f0;
    const size_t pad = f0 * kHop;
    const size_t len = (frames ? frames - 1 : 0) * kHop + kNfft;
    std::vector<double> padded(len);
    for (size_t q = 0; q < len; ++q) {
      const size_t j = pad + q;
      double v = 0.0;
      if (j >= kNfft / 2) {
        const size_t i = j - kNfft / 2;
        if (i == 0)
          v = double(pcm[0]);
        else if (i < n_pcm)
          v = double(pcm[i]) - double(kPreEmphasis) * double(pcm[i - 1]);
      }
      padded[q] = v;
    }
    std::vector<double> frame(kNfft), re(kNfft), im(kNfft);
    std::vector<float> power(kBins);
    for (size_t t = 0; t < frames; ++t) {
      for (size_t i = 0; i < kNfft; ++i) frame[i] = padded[t * kHop + i] * window[i];
      fft.forward(frame.data(), re.data(), im.data());
      for (size_t k = 0; k < kBins; ++k) power[k] = float(re[k] * re[k] + im[k] * im[k]);
      for (size_t m = 0; m < kMels; ++m) {
        float e = 0.0f;
        for (size_t k = spans[m].first; k < spans[m].second; ++k)
          e = std::fma(filters[m * kBins + k], power[k], e);
        out[t * kMels + m] = std::log(e + kLogEps);
      }
    }
  }
};

const Frontend &frontend() {
  static const Frontend f;
  return f;
}

}  // namespace

extern "C" {

// src/fft.rs `Fft::<f64>::new(n).forward(x)`: re and im of n real values.
void wo_fft(const double *x, size_t n, double *re, double *im) { RealFft(n).forward(x, re, im); }

// src/parakeet/frontend.rs:74-108 `Frontend::log_mel(pcm, f0..f1)`: [f1 - f0][128] f32.
void wo_log_mel(const float *pcm, size_t n_pcm, size_t f0, size_t f1, float *out) {
  frontend().log_mel(pcm, n_pcm, f0, f1, out);
}

// src/parakeet/frontend.rs:50-70 `Frontend::compute`: the log-mel of every frame, each mel bin
// normalised over all frames but the last (f64 sums in frame order), the last zero. Returns the
// frames (pcm / 160 + 1), 0 below 3 (nothing written).
size_t wo_mel_features(const float *pcm, size_t n_pcm, float *out) {
  const size_t frames = n_pcm / kHop + 1;
  if (frames < 3) return 0;
  frontend().log_mel(pcm, n_pcm, 0, frames, out);
  const size_t n = frames - 1;
  for (size_t m = 0; m < kMels; ++m) {
    double sum = 0.0;
    for (size_t t = 0; t < n; ++t) sum += double(out[t * kMels + m]);
    const double mean = sum / double(n);
    double var = 0.0;
    for (size_t t = 0; t < n; ++t) {
      const double d = double(out[t * kMels + m]) - mean;
      var += d * d;
    }
    var /= double(n - 1);
    const double inv = 1.0 / (std::sqrt(var) + double(1e-5f));
    for (size_t t = 0; t < n; ++t) out[t * kMels + m] = float((double(out[t * kMels + m]) - mean) * inv);
    out[n * kMels + m] = 0.0f;
  }
  return frames;
}

// The frontend's tables: the Hann window [512] (f64) and the Slaney filterbank [128][257] (f32).
void wo_frontend_tables(double *window, float *filters) {
  const Frontend &f = frontend();
  std::memcpy(window, f.window.data(), kNfft * sizeof(double));
  std::memcpy(filters, f.filters.data(), kMels * kBins * sizeof(float));
}

void wo_set_vnni(int mode) { g_vnni = mode; }
int wo_vnni(void) {
  if (g_vnni < 0) g_vnni = detect_vnni();
  return g_vnni;
}

// src/cpu/gemm.rs:45-75 `Linear::new`: weights [n][k] in a GGUF type (0 F32, 1 F16, 8 Q8_0: blocks
// of an f16 scale and 32 int8), and n biases (NULL for zeros).
void *wo_linear_new(int ty, size_t n, size_t k, const uint8_t *bytes, const float *bias) {
  Linear *l = new Linear();
  l->n = n;
  l->k = k;
  l->ty = ty;
  if (ty == TY_F32) {
    l->f32.resize(n * k);
    std::memcpy(l->f32.data(), bytes, n * k * 4);
  } else if (ty == TY_F16) {
    l->f16.resize(n * k);
    std::memcpy(l->f16.data(), bytes, n * k * 2);
  } else {
    l->q.resize(n * k);
    l->d.resize(n * k / 32);
    for (size_t blk = 0; blk < n * k / 32; ++blk) {
      const uint8_t *b = bytes + 34 * blk;
      l->d[blk] = f16_to_f32(uint16_t(b[0] | (b[1] << 8)));
      std::memcpy(l->q.data() + 32 * blk, b + 2, 32);
    }
  }
  l->bias.assign(n, 0.0f);
  if (bias) std::memcpy(l->bias.data(), bias, n * 4);
  return l;
}

void wo_linear_free(void *l) { delete static_cast<Linear *>(l); }

// src/cpu/gemm.rs:125-177 `gemm`: c = epilogue(a·W^T + b) for m rows of a [m][k] into c [m][n].
// Q8_0 weights on a CPU with VNNI take the i16 path (a quantized per 32 values, exact i32 sums);
// otherwise a and W are rounded to f16 and the f32 tile runs.
void wo_gemm(const float *a, const void *lp, float *c, size_t m, int epi, float alpha) {
  const Linear &l = *static_cast<const Linear *>(lp);
  size_t k = l.k, n = l.n, panels_n = (n + NR - 1) / NR;
  if (l.ty == TY_Q8_0 && wo_vnni() > 0) {
    std::vector<int16_t> aq(m * k);
    std::vector<float> ad(m * k / 32);
    par_each((m + 63) / 64, [&](size_t g) {
      size_t r0 = g * 64, r1 = std::min(m, r0 + 64);
      quantize(a + r0 * k, aq.data() + r0 * k, ad.data() + r0 * k / 32, (r1 - r0) * k / 32);
    });
    size_t blocks = k / 32;
    // One job per (row group, panel group); exact integer sums make the order of products free.
    par_each(panels_n, [&](size_t p) {
      float acc[NR];
      for (size_t r = 0; r < m; ++r) {
        const int16_t *ar = aq.data() + r * k;
        const float *adr = ad.data() + r * blocks;
        size_t cols = std::min(NR, n - NR * p);
        for (size_t j = 0; j < cols; ++j) {
          size_t row = NR * p + j;
          const int8_t *wq = l.q.data() + row * k;
          const float *wd = l.d.data() + row * blocks;
          float s_acc = 0.0f;
          for (size_t blk = 0; blk < blocks; ++blk) {
            __m256i s = _mm256_setzero_si256();
            for (int h = 0; h < 2; ++h) {
              __m256i av = _mm256_loadu_si256((const __m256i *)(ar + 32 * blk + 16 * h));
              __m256i wv = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(wq + 32 * blk + 16 * h)));
              s = _mm256_add_epi32(s, _mm256_madd_epi16(av, wv));
            }
            __m128i s4 = _mm_add_epi32(_mm256_castsi256_si128(s), _mm256_extracti128_si256(s, 1));
            s4 = _mm_add_epi32(s4, _mm_shuffle_epi32(s4, 0x4e));
            s4 = _mm_add_epi32(s4, _mm_shuffle_epi32(s4, 0xb1));
            int32_t sum = _mm_cvtsi128_si32(s4);
            s_acc = std::fma(float(sum), adr[blk] * wd[blk], s_acc);
          }
          acc[j] = s_acc;
        }
        finish(c + r * n + NR * p, acc, l.bias.data() + NR * p, cols, epi, alpha);
      }
    });
    return;
  }
  std::vector<float> ah(m * k);
  for (size_t i = 0; i < m * k; ++i) ah[i] = to_half(a[i]);
  // Groups of panels that fit 384 KiB, then row splits (src/cpu/gemm.rs:223-269).
  size_t bytes = 4 * k * NR;
  size_t per_group = std::min(std::max<size_t>((384u << 10) / bytes, 1), panels_n);
  size_t groups = (panels_n + per_group - 1) / per_group;
  size_t splits = std::max<size_t>(
      std::min((size_t(4 * threads()) + groups - 1) / groups, (m + 8 * MR - 1) / (8 * MR)), 1);
  size_t rows = ceil_to((m + splits - 1) / splits, MR);
  par_each(groups * splits, [&](size_t job) {
    size_t g = job / splits, s = job % splits;
    size_t p0 = g * per_group, p1 = std::min(panels_n, (g + 1) * per_group);
    std::vector<float> buf((p1 - p0) * k * NR);
    for (size_t p = p0; p < p1; ++p) pack_panel(l, p, buf.data() + (p - p0) * k * NR);
    size_t r0 = s * rows, r1 = std::min(m, (s + 1) * rows);
    float acc[MR][NR];
    for (size_t row = r0; row < r1; row += MR) {
      const float *ar[MR];
      for (size_t r = 0; r < MR; ++r) ar[r] = ah.data() + std::min(row + r, r1 - 1) * k;
      for (size_t p = p0; p < p1; ++p) {
        tile(ar, buf.data() + (p - p0) * k * NR, k, acc);
        size_t cols = std::min(NR, n - NR * p);
        for (size_t r = 0; r < MR && row + r < r1; ++r)
          finish(c + (row + r) * n + NR * p, acc[r], l.bias.data() + NR * p, cols, epi, alpha);
      }
    }
  });
}

// src/cpu/gemm.rs:179-208 `gemv`: one row x [k] through the layer in f32 (W not rounded to f16).
void wo_gemv(const float *x, const void *lp, float *c, int epi, float alpha) {
  const Linear &l = *static_cast<const Linear *>(lp);
  size_t k = l.k, n = l.n;
  std::vector<float> acc(n), wide(k);
  for (size_t r = 0; r < n; ++r) {
    if (l.ty == TY_F32) {
      acc[r] = dot(l.f32.data() + r * k, x, k);
    } else if (l.ty == TY_F16) {
      for (size_t i = 0; i < k; ++i) wide[i] = f16_to_f32(l.f16[r * k + i]);
      acc[r] = dot(wide.data(), x, k);
    } else {
      // Q8::rows (src/cpu/mod.rs:412-436): (q · d) rounded to f32 (exact), FMA with x per lane.
      for (size_t i = 0; i < k; ++i) wide[i] = float(l.q[r * k + i]) * l.d[(r * k + i) / 32];
      acc[r] = dot(wide.data(), x, k);
    }
  }
  finish(c, acc.data(), l.bias.data(), n, epi, alpha);
}

}  // extern "C"

// ---- Parakeet's 8x conv subsampling (src/parakeet/cpu.rs:60-174) --------------------------------

namespace {

inline size_t half_up(size_t n) { return (n - 1) / 2 + 1; }  // src/gpu/mod.rs:1068-1070 `half`

// src/parakeet/cpu.rs:151-174 `depthwise`: 3x3, stride 2, padding 1, + bias, over the image
// [t][f][ch] into [half(t)][half(f)][ch]; taps [9][ch] (time tap, then frequency tap). The whole
// image at once (the reference's chunks of rows give the same rows).
void depthwise(const float *x, const float *w, const float *b, size_t t, size_t f, size_t ch,
               float *y, size_t rows) {
  const size_t fo_n = half_up(f);
  for (size_t k = 0; k < rows; ++k)
    for (size_t fo = 0; fo < fo_n; ++fo) {
      float *yy = y + (k * fo_n + fo) * ch;
      for (size_t c = 0; c < ch; ++c) yy[c] = b[c];
      for (size_t tap = 0; tap < 9; ++tap) {
        const size_t ti = 2 * k + tap / 3, fi = 2 * fo + tap % 3;
        if (ti < 1 || ti > t || fi < 1 || fi > f) continue;
        const float *xx = x + ((ti - 1) * f + fi - 1) * ch;
        for (size_t c = 0; c < ch; ++c) yy[c] += w[tap * ch + c] * xx[c];
      }
    }
}

}  // namespace

extern "C" {

// src/parakeet/cpu.rs:60-98 `Encoder::run` up to the conformer: conv0 (3x3 stride 2, 1 -> ch) +
// ReLU over the valid mel frames, conv2 (depthwise) with its rows from half(half(valid)) on zero,
// conv3 (pointwise) + ReLU, conv5 (depthwise), conv6 (pointwise) + ReLU, [t][f][ch] to
// [t][ch * f], and the output projection: x [t][d], t = half(half(half(frames - 1))).
size_t wo_subsample(const float *mel, size_t frames, size_t valid, size_t ch, const float *w0,
                    const float *b0, const float *w2, const float *b2, const void *conv3,
                    const float *w5, const float *b5, const void *conv6, const void *out,
                    float *x) {
  const size_t mels = 128;
  const size_t t1 = half_up(valid), f1 = half_up(mels), f2 = half_up(f1), t2 = half_up(half_up(frames));
  const size_t t = half_up(half_up(half_up(frames - 1))), f = half_up(f2);
  // conv0 + ReLU for rows below t1 (the reference computes them per conv2 row, the same values).
  std::vector<float> c0(t1 * f1 * ch);
  for (size_t r = 0; r < t1; ++r)
    for (size_t c = 0; c < f1; ++c) {
      float *px = c0.data() + (r * f1 + c) * ch;
      for (size_t q = 0; q < ch; ++q) px[q] = b0[q];
      for (size_t tap = 0; tap < 9; ++tap) {
        const size_t tm = 2 * r + tap / 3 - 1, fm = 2 * c + tap % 3 - 1;  // wraps below 0
        const float v = tm < valid && fm < mels ? mel[tm * mels + fm] : 0.0f;
        for (size_t q = 0; q < ch; ++q) px[q] += w0[tap * ch + q] * v;
      }
      for (size_t q = 0; q < ch; ++q) px[q] = std::max(px[q], 0.0f);
    }
  // conv2 over conv0 (rows past t1 zero), its rows from half(t1) on zero.
  std::vector<float> a(t2 * f2 * ch, 0.0f);
  const size_t live = half_up(t1);
  for (size_t k = 0; k < t2 && k < live; ++k)
    for (size_t fo = 0; fo < f2; ++fo) {
      float *yy = a.data() + (k * f2 + fo) * ch;
      for (size_t q = 0; q < ch; ++q) yy[q] = b2[q];
      for (size_t tap = 0; tap < 9; ++tap) {
        const size_t r = 2 * k + tap / 3 - 1;  // conv0 row, wraps below 0
        const size_t c = 2 * fo + tap % 3 - 1;
        if (c >= f1) continue;
        const float *xx = r < t1 ? c0.data() + (r * f1 + c) * ch : nullptr;
        for (size_t q = 0; q < ch; ++q) yy[q] += w2[tap * ch + q] * (xx ? xx[q] : 0.0f);
      }
    }
  std::vector<float> b(a.size());
  wo_gemm(a.data(), conv3, b.data(), t2 * f2, 2 /* relu */, 1.0f);
  std::vector<float> h(t * f * ch);
  depthwise(b.data(), w5, b5, t2, f2, ch, h.data(), t);
  std::vector<float> y(h.size());
  wo_gemm(h.data(), conv6, y.data(), t * f, 2, 1.0f);
  for (size_t r = 0; r < t; ++r)
    for (size_t e = 0; e < f * ch; ++e) h[r * f * ch + e] = y[r * f * ch + (e % f) * ch + e / f];
  wo_gemm(h.data(), out, x, t, 0 /* bias */, 1.0f);
  return t;
}

}  // extern "C"
