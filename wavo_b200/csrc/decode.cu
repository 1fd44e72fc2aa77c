// Decoder-side kernels: the F16 KV-cache pack, split-K attention of one query per head over such a
// cache for a batch of segments, rotary embedding, and the decoder's row projections.
//
// Cache layout (the reference's, decode.wgsl:1-6 and src/gpu/mod.rs:1507-1522): a cache of `cols`
// positions and d dims holds f16 pairs in 32-bit words: K transposed (word i·cols + j is pair i of
// position j), then V by position (word (d/2)·cols + j·(d/2) + i). With K transposed, consecutive
// keys are consecutive words, so the score pass reads K with 16-byte loads across threads.
#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

// ---- pack -------------------------------------------------------------------------------

// rows rows of x (row j: 2·d floats from src + j·stride, K then V) into the cache at positions
// col.. (decode.wgsl:152-173). One thread per (row, pair); rows run fastest so the transposed K
// words of consecutive positions are written together.
__global__ void pack_cache_kernel(const float *__restrict__ x, long long src, long long stride,
                                  uint32_t *__restrict__ cache, int rows, int d, int cols, int col,
                                  long long x_batch, long long cache_batch) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  const long long total = (long long)rows * d;  // d pairs per row (K: d/2, V: d/2)
  const int half = d / 2;
  const float *xb = x + blockIdx.y * x_batch;
  uint32_t *cb = cache + blockIdx.y * cache_batch;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int j = int(t % rows), i = int(t / rows);
    const float *p = xb + src + j * stride + 2LL * i;  // any float offset: two scalar loads
    const float2 v = make_float2(p[0], p[1]);
    const long long at = i < half ? (long long)i * cols + col + j
                                  : (long long)half * cols + (long long)(col + j) * half + (i - half);
    cb[at] = pack_half2(v.x, v.y);
  }
}

// ---- attend -----------------------------------------------------------------------------

constexpr int ATT_THREADS = 256;
constexpr int ATT_KEYS = 1024;  // keys per CTA: 4 per thread with 16-byte loads

__device__ __forceinline__ float block_reduce(float v, float *red, bool is_max) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int i = 1; i < ATT_THREADS / 32; ++i) v = is_max ? fmaxf(v, red[i]) : v + red[i];
  return v;
}

__device__ __forceinline__ float2 h2f(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2 *>(&w);
  return __half22float2(h);
}

// CTA (split, head, segment): keys split·ATT_KEYS .. of head h of segment b. Writes the partial
// (Σ e·V, m, l) to part, or with one split the normalised output directly.
__global__ void __launch_bounds__(ATT_THREADS, 5)
    attend_kernel(const float *__restrict__ q, long long q_stride, const uint32_t *__restrict__ kv,
                  long long kv_stride, float *__restrict__ part, float *__restrict__ o,
                  long long o_stride, int n, int cols, int hd, float scale) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  __shared__ float qs[128];
  __shared__ float ps[ATT_KEYS];
  __shared__ float red[ATT_THREADS / 32];
  __shared__ float acc_s[ATT_THREADS / 8 * 64 + 64];
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int splits = gridDim.x, heads = gridDim.y;
  const int pairs = hd / 2;
  const int d = heads * hd;
  const uint32_t *cache = kv + b * kv_stride;
  const uint32_t *kt = cache + (long long)h * pairs * cols;       // K^T rows of this head
  const uint32_t *vv = cache + (long long)(d / 2) * cols + h * pairs;  // V, stride d/2 words
  for (int i = threadIdx.x; i < hd; i += ATT_THREADS)
    qs[i] = __half2float(__float2half_rn(q[b * q_stride + h * hd + i]));
  __syncthreads();

  const int j0 = split * ATT_KEYS;
  const int nk = min(ATT_KEYS, n - j0);
  // Scores: thread t takes keys j0 + 4t .. 4t + 3.
  float sc[4];
  float mx = -INFINITY;
  const int jt = 4 * threadIdx.x;
  const bool aligned = ((kv_stride & 3) == 0) && ((reinterpret_cast<uintptr_t>(kv) & 15u) == 0);
  const bool vec = aligned && ((cols & 3) == 0);
#pragma unroll
  for (int u = 0; u < 4; ++u) sc[u] = 0.0f;
  if (vec && nk <= 4 * (ATT_THREADS / 4)) {
    // At most 256 keys (a decoder's self-attention): thread t takes key quad t % 64 over a quarter
    // of the pairs (8 at hd 64), its loads issued four at a time; the quarters meet in ps.
    const int kq = threadIdx.x % (ATT_THREADS / 4), pg = threadIdx.x / (ATT_THREADS / 4);
    const int jq = 4 * kq, ppg = (pairs + 3) / 4;
    const int i0 = pg * ppg, i1 = min(pairs, i0 + ppg);
    float pa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (jq < nk) {
      for (int i = i0; i < i1; i += 4) {
        uint32_t w[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (i + u >= i1) break;
          const uint32_t *row = kt + (long long)(i + u) * cols + j0 + jq;
          if (jq + 3 < nk) {
            const uint4 x = *reinterpret_cast<const uint4 *>(row);
            w[u][0] = x.x; w[u][1] = x.y; w[u][2] = x.z; w[u][3] = x.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) w[u][e] = jq + e < nk ? row[e] : 0u;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (i + u >= i1) break;
          const float q0 = qs[2 * (i + u)], q1 = qs[2 * (i + u) + 1];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 k = h2f(w[u][e]);
            pa[e] = fmaf(q1, k.y, fmaf(q0, k.x, pa[e]));
          }
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ps[pg * (ATT_KEYS / 4) + jq + e] = pa[e];
    __syncthreads();
    if (jt < nk) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        sc[e] = ps[jt + e] + ps[ATT_KEYS / 4 + jt + e] + ps[2 * (ATT_KEYS / 4) + jt + e] +
                ps[3 * (ATT_KEYS / 4) + jt + e];
    }
    __syncthreads();  // ps is rewritten with the probabilities below
  } else if (jt < nk) {
    if (vec && jt + 3 < nk) {
      for (int i = 0; i < pairs; ++i) {
        const uint4 w = *reinterpret_cast<const uint4 *>(kt + (long long)i * cols + j0 + jt);
        const float q0 = qs[2 * i], q1 = qs[2 * i + 1];
        float2 k;
        k = h2f(w.x); sc[0] = fmaf(q1, k.y, fmaf(q0, k.x, sc[0]));
        k = h2f(w.y); sc[1] = fmaf(q1, k.y, fmaf(q0, k.x, sc[1]));
        k = h2f(w.z); sc[2] = fmaf(q1, k.y, fmaf(q0, k.x, sc[2]));
        k = h2f(w.w); sc[3] = fmaf(q1, k.y, fmaf(q0, k.x, sc[3]));
      }
    } else {
      for (int i = 0; i < pairs; ++i) {
        const uint32_t *row = kt + (long long)i * cols + j0 + jt;
        const float q0 = qs[2 * i], q1 = qs[2 * i + 1];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (jt + u < nk) {
            float2 k = h2f(row[u]);
            sc[u] = fmaf(q1, k.y, fmaf(q0, k.x, sc[u]));
          }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    sc[u] = (jt + u < nk) ? sc[u] * scale : -INFINITY;
    mx = fmaxf(mx, sc[u]);
  }
  const float m = block_reduce(mx, red, true);
  float lsum = 0.0f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float e = (jt + u < nk) ? __expf(sc[u] - m) : 0.0f;
    if (jt + u < ATT_KEYS) ps[jt + u] = e;
    lsum += e;
  }
  const float l = block_reduce(lsum, red, false);
  __syncthreads();

  // P·V: thread (g, c4): 4 consecutive pairs c4..c4+3 of keys g, g + G, ... (G = threads / (pairs/4)).
  const int quads = pairs / 4;  // hd % 8 == 0 for this path
  float acc[8];
#pragma unroll
  for (int x = 0; x < 8; ++x) acc[x] = 0.0f;
  if (aligned && quads > 0 && (pairs & 3) == 0 && ((d / 2) & 3) == 0) {
    const int groups = ATT_THREADS / quads;
    const int g = threadIdx.x / quads, c4 = threadIdx.x % quads;
    if (g < groups) {
      for (int jj = g; jj < nk; jj += groups) {
        const uint4 w =
            *reinterpret_cast<const uint4 *>(vv + (long long)(j0 + jj) * (d / 2) + 4 * c4);
        const float e = ps[jj];
        float2 v;
        v = h2f(w.x); acc[0] = fmaf(e, v.x, acc[0]); acc[1] = fmaf(e, v.y, acc[1]);
        v = h2f(w.y); acc[2] = fmaf(e, v.x, acc[2]); acc[3] = fmaf(e, v.y, acc[3]);
        v = h2f(w.z); acc[4] = fmaf(e, v.x, acc[4]); acc[5] = fmaf(e, v.y, acc[5]);
        v = h2f(w.w); acc[6] = fmaf(e, v.x, acc[6]); acc[7] = fmaf(e, v.y, acc[7]);
      }
    }
    // Reduce over the groups through shared memory: acc_s[g][8·c4 + x].
    __syncthreads();
    if (g < groups)
#pragma unroll
      for (int x = 0; x < 8; ++x) acc_s[g * hd + 8 * c4 + x] = acc[x];
    __syncthreads();
    for (int c = threadIdx.x; c < hd; c += ATT_THREADS) {
      float t = 0.0f;
      for (int gg = 0; gg < groups; ++gg) t += acc_s[gg * hd + c];
      if (splits == 1) {
        o[b * o_stride + h * hd + c] = t / l;
      } else {
        part[(((long long)b * heads + h) * splits + split) * (hd + 2) + c] = t;
      }
    }
  } else {
    // Scalar path for heads whose pairs do not come in fours.
    for (int c = threadIdx.x; c < pairs; c += ATT_THREADS) {
      float t0 = 0.0f, t1 = 0.0f;
      for (int jj = 0; jj < nk; ++jj) {
        const float2 v = h2f(vv[(long long)(j0 + jj) * (d / 2) + c]);
        t0 = fmaf(ps[jj], v.x, t0);
        t1 = fmaf(ps[jj], v.y, t1);
      }
      if (splits == 1) {
        o[b * o_stride + h * hd + 2 * c] = t0 / l;
        o[b * o_stride + h * hd + 2 * c + 1] = t1 / l;
      } else {
        float *pp = part + (((long long)b * heads + h) * splits + split) * (hd + 2);
        pp[2 * c] = t0;
        pp[2 * c + 1] = t1;
      }
    }
  }
  if (splits > 1 && threadIdx.x == 0) {
    float *pp = part + (((long long)b * heads + h) * splits + split) * (hd + 2);
    pp[hd] = m;
    pp[hd + 1] = l;
  }
}

// One CTA per (head, segment): the parts rescaled to their common maximum, summed, normalised
// (decode.wgsl:124-147).
__global__ void combine_kernel(const float *__restrict__ part, float *__restrict__ o,
                               long long o_stride, int splits, int hd) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  const int h = blockIdx.x, b = blockIdx.y, heads = gridDim.x;
  const float *base = part + ((long long)b * heads + h) * splits * (hd + 2);
  float m = -INFINITY;
  for (int c = 0; c < splits; ++c) m = fmaxf(m, base[c * (hd + 2) + hd]);
  float l = 0.0f;
  for (int c = 0; c < splits; ++c) l += __expf(base[c * (hd + 2) + hd] - m) * base[c * (hd + 2) + hd + 1];
  for (int i = threadIdx.x; i < hd; i += blockDim.x) {
    float t = 0.0f;
    for (int c = 0; c < splits; ++c) t += __expf(base[c * (hd + 2) + hd] - m) * base[c * (hd + 2) + i];
    o[b * o_stride + h * hd + i] = t / l;
  }
}

// ---- rope ------------------------------------------------------------------------------

// In place over rows of `stride` elements: heads 0 .. sections·heads - 1 of hd dims rotate their
// pairs (2i, 2i+1), or with neox (i, i + rot/2), for 2i < rot, by table row pos + row (rot/2
// cosines then rot/2 sines) (ops.wgsl:191-215, src/cpu/ops.rs:339-355).
template <typename T>
__global__ void rope_kernel(const float *__restrict__ table, T *__restrict__ x, long long stride,
                            int rows, int pos, const int *__restrict__ positions, int heads, int hd,
                            int rot, int neox, int sections) {
  const int half = rot / 2;
  const long long per_row = (long long)sections * heads * half;
  const long long total = per_row * rows;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int r = int(t / per_row);
    const int rem = int(t % per_row);
    const int hh = rem / half, i = rem % half;
    const long long at = positions ? positions[r] : pos + r;  // the row's table row
    const float c = table[at * rot + i], s = table[at * rot + half + i];
    T *head = x + r * stride + (long long)hh * hd;
    const int i0 = neox ? i : 2 * i, i1 = neox ? i + half : 2 * i + 1;
    const float a = float(head[i0]), b = float(head[i1]);
    head[i0] = T(a * c - b * s);
    head[i1] = T(a * s + b * c);
  }
}

// f16 rows, four rotary pairs a thread (half = rot / 2 a multiple of 4, 8-byte aligned heads):
// one row per grid row, the row's cos / sin read as float4, the pairs as 8- or 16-byte words.
__device__ __forceinline__ void rot2(float a, float b, float c, float s, __half &x0, __half &x1) {
  x0 = __float2half_rn(a * c - b * s);
  x1 = __float2half_rn(a * s + b * c);
}

__global__ void rope4_kernel(const float *__restrict__ table, __half *__restrict__ x,
                             long long stride, int rows, int pos, const int *__restrict__ positions,
                             int heads, int hd, int rot, int neox, int sections) {
  const int half = rot / 2, q4 = half / 4;
  const int per_row = sections * heads * q4;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const long long at = positions ? positions[r] : pos + (long long)r;
    const float *cs = table + at * rot;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < per_row; t += gridDim.x * blockDim.x) {
      const int hh = t / q4, i = (t - hh * q4) * 4;
      __half *head = x + (long long)r * stride + (long long)hh * hd;
      const float4 c = *reinterpret_cast<const float4 *>(cs + i);
      const float4 sn = *reinterpret_cast<const float4 *>(cs + half + i);
      const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
      if (neox) {  // pairs (i + k, i + k + half)
        uint2 lo = *reinterpret_cast<const uint2 *>(head + i);
        uint2 hi = *reinterpret_cast<const uint2 *>(head + i + half);
        __half *l = reinterpret_cast<__half *>(&lo), *u = reinterpret_cast<__half *>(&hi);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          rot2(__half2float(l[k]), __half2float(u[k]), cc[k], ss[k], l[k], u[k]);
        *reinterpret_cast<uint2 *>(head + i) = lo;
        *reinterpret_cast<uint2 *>(head + i + half) = hi;
      } else {  // pairs (2(i + k), 2(i + k) + 1)
        uint4 w = *reinterpret_cast<const uint4 *>(head + 2 * i);
        __half *e = reinterpret_cast<__half *>(&w);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          rot2(__half2float(e[2 * k]), __half2float(e[2 * k + 1]), cc[k], ss[k], e[2 * k],
               e[2 * k + 1]);
        *reinterpret_cast<uint4 *>(head + 2 * i) = w;
      }
    }
  }
}

// ---- gemv ------------------------------------------------------------------------------

// c[r][n] = epilogue(Σ_k a[r][k]·W[n][k] + bias[n]) for r < rows, in f32 (W f16 exact), one warp
// per output feature; the row rounding of the reference's gemv (none) is kept.
constexpr int GEMV_ROWS = 32;

__device__ __forceinline__ float gelu_g(float x) {
  float z = fabsf(0.70710678118654752f * x);
  float t = 1.0f / (1.0f + 0.3275911f * z);
  float p = (((1.0614054f * t - 1.453152f) * t + 1.4214138f) * t - 0.28449674f) * t + 0.2548296f;
  float s = signbit(x) ? -1.0f : 1.0f;
  return 0.5f * x * (1.0f + s * (1.0f - p * t * expf(-z * z)));
}

template <int WT>
__device__ __forceinline__ void load_w8(const void *w, const float *scales, long long f, int k,
                                        int k0, float (&wf)[8]) {
  if (WT == 1) {
    const uint4 wv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(w) + f * k + k0);
    float2 t;
    t = h2f(wv.x); wf[0] = t.x; wf[1] = t.y;
    t = h2f(wv.y); wf[2] = t.x; wf[3] = t.y;
    t = h2f(wv.z); wf[4] = t.x; wf[5] = t.y;
    t = h2f(wv.w); wf[6] = t.x; wf[7] = t.y;
  } else if (WT == 0) {
    const float *p = reinterpret_cast<const float *>(w) + f * k + k0;
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
    wf[0] = a.x; wf[1] = a.y; wf[2] = a.z; wf[3] = a.w;
    wf[4] = b.x; wf[5] = b.y; wf[6] = b.z; wf[7] = b.w;
  } else {
    const int8_t *p = reinterpret_cast<const int8_t *>(w) + f * k + k0;
    const uint2 q = *reinterpret_cast<const uint2 *>(p);
    const float d = scales[(f * k + k0) / 32];
    const int8_t *qb = reinterpret_cast<const int8_t *>(&q);
#pragma unroll
    for (int i = 0; i < 8; ++i) wf[i] = float(qb[i]) * d;  // exact in f32, as Q8::rows
  }
}

template <int WT>
__global__ void __launch_bounds__(256)
    gemv_kernel(const float *__restrict__ a, long long lda, const void *__restrict__ w,
                const float *__restrict__ scales, const float *__restrict__ bias,
                float *__restrict__ c, long long ldc, int rows, int n, int k, int epi, float alpha) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f = blockIdx.x * 8 + warp;
  if (f >= n) return;
  float acc[GEMV_ROWS];
#pragma unroll
  for (int r = 0; r < GEMV_ROWS; ++r) acc[r] = 0.0f;
  for (int k0 = 8 * lane; k0 < k; k0 += 256) {
    float wf[8];
    load_w8<WT>(w, scales, f, k, k0, wf);
#pragma unroll
    for (int r = 0; r < GEMV_ROWS; ++r) {
      if (r < rows) {
        const float4 x0 = *reinterpret_cast<const float4 *>(a + r * lda + k0);
        const float4 x1 = *reinterpret_cast<const float4 *>(a + r * lda + k0 + 4);
        float s = acc[r];
        s = fmaf(x0.x, wf[0], s); s = fmaf(x0.y, wf[1], s); s = fmaf(x0.z, wf[2], s);
        s = fmaf(x0.w, wf[3], s); s = fmaf(x1.x, wf[4], s); s = fmaf(x1.y, wf[5], s);
        s = fmaf(x1.z, wf[6], s); s = fmaf(x1.w, wf[7], s);
        acc[r] = s;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < GEMV_ROWS; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  }
  if (lane < rows) {
    float v = 0.0f;
#pragma unroll
    for (int r = 0; r < GEMV_ROWS; ++r)
      if (r == lane) v = acc[r];
    v += bias[f];
    float *cp = c + lane * ldc + f;
    switch (epi) {
      case kBias: *cp = v; break;
      case kSilu: *cp = v / (1.0f + expf(-v)); break;
      case kRelu: *cp = fmaxf(v, 0.0f); break;
      case kResidual: *cp += alpha * v; break;
      case kGelu: *cp = gelu_g(v); break;
      case kGeluResidual: *cp += gelu_g(v); break;
      default: *cp = tanhf(fminf(fmaxf(v, -10.0f), 10.0f)); break;
    }
  }
}


// Split-K form for the bias and residual epilogues: a CTA takes 64 output features and a range of
// k; its W tile goes to shared memory once (as f32: W f16 exact, Q8_0 as q·d exact); lane r of a
// warp is row r and holds 32 of its k values of a in registers, reused over the warp's 8 features
// (each W value a shared-memory broadcast). Partial sums go to c with f32 atomics: c += alpha ·
// (sum + bias) for the residual epilogue; for the bias epilogue c is cleared first and gets
// sum + bias. (The full-k kernel above re-reads the rows of a for every feature.)
constexpr int GS_F = 64;   // features per CTA
constexpr int GS_KC = 32;  // k per register chunk

template <int WT>
__global__ void __launch_bounds__(256)
    gemv_split_kernel(const float *__restrict__ a, long long lda, const void *__restrict__ w,
                      const float *__restrict__ scales, const float *__restrict__ bias,
                      float *__restrict__ c, long long ldc, int rows, int n, int k, int kr,
                      int epi, float alpha) {
  extern __shared__ float4 ws4[];
  float *ws = reinterpret_cast<float *>(ws4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * GS_F, k0 = blockIdx.y * kr;
  const int kn = min(kr, k - k0);  // a multiple of 32 (k and kr are)
  // W tile [64][kr] as f32: every load of the tile in flight at once (one memory latency), then
  // the conversions and shared-memory stores.
  constexpr int IT = GS_F * 256 / (256 * 8);  // loads of 8 values per thread (kr <= 256)
  float wf[IT][8];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int i = (it * 256 + threadIdx.x) * 8;
    const int f = i / kr, kk = i - f * kr;
    if (i < GS_F * kr && f0 + f < n && kk < kn) {
      load_w8<WT>(w, scales, f0 + f, k, k0 + kk, wf[it]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wf[it][j] = 0.0f;
    }
  }
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int i = (it * 256 + threadIdx.x) * 8;
    if (i < GS_F * kr) {
      *reinterpret_cast<float4 *>(ws + i) = make_float4(wf[it][0], wf[it][1], wf[it][2], wf[it][3]);
      *reinterpret_cast<float4 *>(ws + i + 4) =
          make_float4(wf[it][4], wf[it][5], wf[it][6], wf[it][7]);
    }
  }
  __syncthreads();
  float acc[8];
#pragma unroll
  for (int f = 0; f < 8; ++f) acc[f] = 0.0f;
  const bool live = lane < rows;
  const float *arow = a + (long long)lane * lda + k0;
  for (int kc = 0; kc < kn; kc += GS_KC) {
    float av[GS_KC];
#pragma unroll
    for (int j = 0; j < GS_KC; j += 4) {
      const float4 t = live ? *reinterpret_cast<const float4 *>(arow + kc + j)
                            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      av[j] = t.x;
      av[j + 1] = t.y;
      av[j + 2] = t.z;
      av[j + 3] = t.w;
    }
#pragma unroll
    for (int f = 0; f < 8; ++f) {
      const float *wr = ws + (warp * 8 + f) * kr + kc;
      float sacc = acc[f];
#pragma unroll
      for (int j = 0; j < GS_KC; j += 4) {
        const float4 wv = *reinterpret_cast<const float4 *>(wr + j);
        sacc = fmaf(av[j], wv.x, sacc);
        sacc = fmaf(av[j + 1], wv.y, sacc);
        sacc = fmaf(av[j + 2], wv.z, sacc);
        sacc = fmaf(av[j + 3], wv.w, sacc);
      }
      acc[f] = sacc;
    }
  }
  if (!live) return;
#pragma unroll
  for (int f = 0; f < 8; ++f) {
    const int feat = f0 + warp * 8 + f;
    if (feat >= n) break;
    float v = acc[f];
    if (blockIdx.y == 0) v += bias[feat];
    atomicAdd(c + (long long)lane * ldc + feat, epi == kResidual ? alpha * v : v);
  }
}


// ---- gemv on the tensor core (F16 weights) -------------------------------------------------
//
// c[r][f] = epilogue(Σ_k a[r][k]·W[f][k] + bias[f]) for rows r < rows (at most 32), W f16 [n][k].
// The rows of a are split exactly enough for f32 accuracy: a = hi + lo with hi = f16(a), lo =
// f16(a - hi) (|a - hi - lo| <= 2^-22 |a|). The product is taken transposed, D = W · X^T: W's 128
// features of a tile are the UMMA's M = 128 rows (the A operand, straight from W's TMA tiles) and
// X = [hi rows 0-31; lo rows 32-63] is the N = 64 operand, so that no UMMA row is wasted and TMEM
// lane f holds feature f with hi·W in columns 0-31 and lo·W in columns 32-63: each epilogue thread
// owns one feature of all 32 rows and adds its two halves in registers.
//
// Both operands arrive by TMA through rings, k outermost: for each 64-column chunk of k the CTA
// loads the rows of a as an f32 [32][64] box (zero fill past `rows` and k) into an X slot, where
// one warp converts it in place to the hi/lo rows in the UMMA's 128-byte swizzle, and then streams
// the W chunk of each of its tiles (up to 8, one 64-column TMEM accumulator each). X needs only a
// few slots, and the rest of shared memory goes to the W ring, deep enough to keep HBM busy. (Plain
// loads of a, replicated over every CTA, are limited by the small L1 that the large shared-memory
// carve-out leaves: few lines in flight per SM. TMA is not.)
//
// Work split: with at least about one 128-feature tile per SM (the logits over a vocabulary) each
// CTA takes tiles blockIdx.x, + gridDim.x, ... with the whole k. With fewer tiles, k is split over
// a cluster of up to 8 CTAs (one tile each): the CTAs stage their partial sums in shared memory and
// CTA q finishes rows q, q + ks, ..., adding every CTA's partials (read through distributed shared
// memory) in rank order, so that every epilogue (GELU, SiLU, the residual add) sees the whole sum
// and the result does not depend on timing. The epilogue is a template parameter: one small body
// per kernel, unrolled over the 32 rows.
//
// Roles (256 threads): warp 4 lane 0 loads W, warp 7 lane 0 loads the rows of a, warp 5 lane 0
// issues the UMMAs, warps 0-3 (TMEM subpartitions 0-3) convert the X chunks (warp s those of slot s,
// so that each waits on its slot's phases in order) and then run the epilogue. The W loads that fit
// the ring do not depend on the previous kernel of the stream and start before griddepcontrol.wait.
constexpr int GT_N = 128;           // features per tile (UMMA M)
constexpr int GT_TMAX = 8;          // tiles per CTA (8 x 64 TMEM columns)
constexpr int GT_THREADS = 256;
constexpr int GT_MAX_CLUSTER = 8;   // portable cluster size
constexpr int GT_XS = 4;            // X slots
constexpr int GT_MAX_STAGES = 12;   // W ring slots
constexpr int GT_SMEM_MAX = 232448; // 227 KB per CTA
constexpr uint32_t GT_X_CHUNK = 8192, GT_W_CHUNK = 16384;

struct __align__(8) GtBarriers {
  uint64_t full[GT_MAX_STAGES];
  uint64_t empty[GT_MAX_STAGES];
  uint64_t x_loaded[GT_XS];  // the f32 box of the slot's X chunk landed
  uint64_t x_ready[GT_XS];   // converted (hi/lo, swizzled)
  uint64_t x_empty[GT_XS];   // the UMMAs of every tile are done with it
  uint64_t acc_full;         // every UMMA of the CTA completed
  uint32_t tmem_base;
  uint32_t abort;
};

__host__ __device__ constexpr size_t gt_smem_bytes(int stages) {
  return 1024 + size_t(GT_XS) * GT_X_CHUNK + size_t(stages) * GT_W_CHUNK + sizeof(GtBarriers);
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

template <int EPI>
__device__ __forceinline__ float gemv_epilogue(float v, float old, float alpha) {
  if constexpr (EPI == kBias) return v;
  else if constexpr (EPI == kSilu) return v / (1.0f + expf(-v));
  else if constexpr (EPI == kRelu) return fmaxf(v, 0.0f);
  else if constexpr (EPI == kResidual) return old + alpha * v;
  else if constexpr (EPI == kGelu) return gelu_g(v);
  else if constexpr (EPI == kGeluResidual) return old + gelu_g(v);
  else return tanhf(fminf(fmaxf(v, -10.0f), 10.0f));
}

// X chunk in place: the f32 box [32 rows][64] (256-byte rows, as TMA wrote it) becomes hi rows 0-31
// and lo rows 32-63 of 128 bytes in the 128-byte swizzle. Lane l takes the 16-byte units l % 8 of
// rows l / 8, l / 8 + 4, ...: every value is read into registers before the warp writes any.
__device__ __forceinline__ void gt_convert_chunk(uint8_t *slot, uint32_t lane) {
  const int u = int(lane & 7);
  float4 v[8][2];
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + int(lane >> 3);
    const float4 *src = reinterpret_cast<const float4 *>(slot + r * 256 + u * 32);
    v[it][0] = src[0];
    v[it][1] = src[1];
  }
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + int(lane >> 3);
    const float x[8] = {v[it][0].x, v[it][0].y, v[it][0].z, v[it][0].w,
                        v[it][1].x, v[it][1].y, v[it][1].z, v[it][1].w};
    float lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) lo[e] = x[e] - __half2float(__float2half_rn(x[e]));
    const int off = (u ^ (r & 7)) << 4;
    *reinterpret_cast<uint4 *>(slot + r * 128 + off) =
        make_uint4(pack_half2(x[0], x[1]), pack_half2(x[2], x[3]), pack_half2(x[4], x[5]),
                   pack_half2(x[6], x[7]));
    *reinterpret_cast<uint4 *>(slot + (r + 32) * 128 + off) =
        make_uint4(pack_half2(lo[0], lo[1]), pack_half2(lo[2], lo[3]), pack_half2(lo[4], lo[5]),
                   pack_half2(lo[6], lo[7]));
  }
}

template <int EPI>
__global__ void __launch_bounds__(GT_THREADS, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                   const __grid_constant__ CUtensorMap map_a, const float *__restrict__ bias,
                   float *__restrict__ c, long long ldc, int rows, int n, int k, int kr,
                   int stages, int tiles, float alpha, int *err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  constexpr bool kReadsC = EPI == kResidual || EPI == kGeluResidual;
  const int ks = int(gridDim.y);  // CTAs of a cluster along k (1: the whole k)
  const int k0 = int(blockIdx.y) * kr;
  const int kn = min(kr, k - k0);
  const int nch = (kn + 63) / 64;
  uint8_t *sx = smem;                             // X slots: [GT_XS][8 KB]
  uint8_t *sw = smem + GT_XS * GT_X_CHUNK;        // W ring: [stages][128 features][128 B]
  GtBarriers *bar = reinterpret_cast<GtBarriers *>(sw + stages * GT_W_CHUNK);
  const uint32_t warp = warp_id(), lane = lane_id();
  // This CTA's tiles: blockIdx.x + t·gridDim.x for t < T (one when k is split; at most GT_TMAX).
  const int T = ks > 1 ? 1 : (tiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
  const int total = nch * T;  // W chunks g = ch·T + t
  const uint32_t tcols = T <= 2 ? 128u : T <= 4 ? 256u : 512u;
  // The CTA's chunks in a rotated order (chunk ch is k column k0 + 64·((ch + rot) mod nch)), so that
  // the CTAs do not all ask L2 for the same rows of a at once.
  const int rot = int(blockIdx.x) % nch;
  const auto kchunk = [&](int ch) { return k0 + ((ch + rot) % nch) * 64; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    for (int s = 0; s < GT_XS; ++s) {
      mbar_init(&bar->x_loaded[s], 1);
      mbar_init(&bar->x_ready[s], 1);
      mbar_init(&bar->x_empty[s], 1);
    }
    mbar_init(&bar->acc_full, 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&bar->tmem_base, tcols);  // one accumulator of 64 columns a tile
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch_dependents();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, err};
  const int pre = total < stages ? total : stages;
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&map_w);
    for (int g = 0; g < pre; ++g) {  // W does not wait for the previous kernel of the stream
      const int slot = g % stages;
      mbar_arrive_expect_tx(&bar->full[slot], GT_W_CHUNK);
      tma_load_2d(sw + slot * GT_W_CHUNK, &map_w, &bar->full[slot], kchunk(g / T),
                  (int(blockIdx.x) + (g % T) * int(gridDim.x)) * GT_N);
    }
  }
  griddep_wait();  // the previous kernel of the stream has completed (a and c are ready)

  if (warp == 4) {
    if (lane == 0) {  // W producer
#pragma unroll 1
      for (int g = pre; g < total; ++g) {
        const int slot = g % stages;
        if (!mbar_wait(&bar->empty[slot], ((g / stages) - 1) & 1, ab, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&bar->full[slot], GT_W_CHUNK);
        tma_load_2d(sw + slot * GT_W_CHUNK, &map_w, &bar->full[slot], kchunk(g / T),
                    (int(blockIdx.x) + (g % T) * int(gridDim.x)) * GT_N);
      }
    }
  } else if (warp == 7) {
    if (lane == 0) {  // X producer: the rows of a, chunk by chunk
      prefetch_tmap(&map_a);
#pragma unroll 1
      for (int ch = 0; ch < nch; ++ch) {
        const int s = ch % GT_XS;
        if (ch >= GT_XS &&
            !mbar_wait(&bar->x_empty[s], ((ch / GT_XS) - 1) & 1, ab, kErrTimeoutProducer))
          break;
        mbar_arrive_expect_tx(&bar->x_loaded[s], GT_X_CHUNK);
        tma_load_2d(sx + s * GT_X_CHUNK, &map_a, &bar->x_loaded[s], kchunk(ch), 0);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // UMMA issuer
      const uint64_t dx0 = sdesc_sw128(smem_u32(sx), 16, 1024);
      const uint64_t dw0 = sdesc_sw128(smem_u32(sw), 16, 1024);
      constexpr uint32_t IDESC = idesc_f16(128, 64, 0);
      bool ok = true;
#pragma unroll 1
      for (int ch = 0; ch < nch && ok; ++ch) {
        const int s = ch % GT_XS;
        if (!mbar_wait(&bar->x_ready[s], (ch / GT_XS) & 1, ab, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        const uint64_t dx = dx0 + uint64_t((s * GT_X_CHUNK) >> 4);
#pragma unroll 1
        for (int t = 0; t < T; ++t) {
          const int g = ch * T + t;
          const int slot = g % stages;
          if (!mbar_wait(&bar->full[slot], (g / stages) & 1, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t dw = dw0 + uint64_t((slot * GT_W_CHUNK) >> 4);
          const uint32_t d = tmem + uint32_t(t * 64);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 16 columns of k = 32 bytes a step
            umma_f16(d, dw + 2 * kk, dx + 2 * kk, IDESC, (ch > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&bar->empty[slot]);
        }
        umma_commit(&bar->x_empty[s]);
      }
      if (ok) umma_commit(&bar->acc_full);
    }
  } else if (warp < 4) {
    // Converters: warp s takes the chunks of X slot s.
#pragma unroll 1
    for (int ch = int(warp); ch < nch; ch += GT_XS) {
      const int s = ch % GT_XS;
      if (!mbar_wait_warp(&bar->x_loaded[s], (ch / GT_XS) & 1, ab, kErrTimeoutConsumer)) break;
      gt_convert_chunk(sx + s * GT_X_CHUNK, lane);
      fence_proxy_async_smem();  // the UMMAs read the chunk through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->x_ready[s]);
    }
  }
  float *part = reinterpret_cast<float *>(sx);  // split k: this CTA's partials [32][128] (X is free)
  if (warp < 4) {
    // Epilogue: lane l of warp w is feature 32w + l of each tile; TMEM columns 64t .. 64t + 31
    // hold its hi·W of rows 0-31 for tile t, the next 32 its lo·W.
    const int fl = int(warp) * 32 + int(lane);
    // The bias of every tile, loaded while the UMMAs run (a load per tile after them would expose
    // its latency each time).
    float bt[GT_TMAX];
#pragma unroll
    for (int t = 0; t < GT_TMAX; ++t) {
      const int f = (int(blockIdx.x) + t * int(gridDim.x)) * GT_N + fl;
      bt[t] = ks == 1 && t < T && f < n ? bias[f] : 0.0f;
    }
    if (mbar_wait_warp(&bar->acc_full, 0, ab, kErrTimeoutConsumer)) {
      tc_fence_after();
#pragma unroll 1
      for (int t = 0; t < T; ++t) {
        uint32_t hi[32], lo[32];
        const uint32_t taddr = tmem + ((warp * 32u) << 16) + uint32_t(t * 64);
        tmem_ld32(taddr, hi);
        tmem_ld32(taddr + 32, lo);
        tmem_wait_ld();
        if (ks == 1) {
          const int f = (int(blockIdx.x) + t * int(gridDim.x)) * GT_N + fl;
          if (f < n) {
            float b = bt[0];
#pragma unroll
            for (int q = 1; q < GT_TMAX; ++q)
              if (q == t) b = bt[q];
#pragma unroll
            for (int r = 0; r < 32; ++r) {
              if (r < rows) {
                float *cp = c + (long long)r * ldc + f;
                const float v = (__uint_as_float(hi[r]) + __uint_as_float(lo[r])) + b;
                *cp = gemv_epilogue<EPI>(v, kReadsC ? *cp : 0.0f, alpha);
              }
            }
          }
        } else {
#pragma unroll
          for (int r = 0; r < 32; ++r)
            part[r * GT_N + fl] = __uint_as_float(hi[r]) + __uint_as_float(lo[r]);
        }
      }
    }
  }
  if (ks > 1) {
    // Every CTA of the cluster has its partials in shared memory; CTA q finishes rows q, q + ks, ...
    // (threads 0-127 and 128-255 take alternate ones), adding the CTAs' partials in rank order.
    __syncwarp();
    cluster_sync();
    const uint32_t rank = cluster_ctarank();
    const int fl = int(threadIdx.x) & (GT_N - 1);
    const int f = int(blockIdx.x) * GT_N + fl;
    if (f < n) {
      const float b = bias[f];
#pragma unroll 1
      for (int r = int(rank) + ks * int(threadIdx.x >> 7); r < rows; r += 2 * ks) {
        float p8[GT_MAX_CLUSTER];
#pragma unroll
        for (int p = 0; p < GT_MAX_CLUSTER; ++p)
          p8[p] = p < ks ? ld_cluster_f32(mapa_shared(part + r * GT_N + fl, uint32_t(p))) : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (int p = 0; p < GT_MAX_CLUSTER; ++p) v += p8[p];
        v += b;
        float *cp = c + (long long)r * ldc + f;
        *cp = gemv_epilogue<EPI>(v, kReadsC ? *cp : 0.0f, alpha);
      }
    }
    __syncwarp();
    cluster_sync();  // the peers' shared memory stays until every CTA has read it
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, tcols);
}

}  // namespace

cudaError_t launch_pack_cache(const float *x, long long src, long long stride, uint32_t *cache,
                              int rows, int d, int cols, int col, long long x_batch,
                              long long cache_batch, int batch, cudaStream_t s) {
  const long long total = (long long)rows * d;
  if (total <= 0 || batch <= 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  return launch_pdl(pack_cache_kernel, dim3(int(blocks), batch), dim3(256), 0, s, x, src, stride,
                    cache, rows, d, cols, col, x_batch, cache_batch);
}

size_t attend_part_floats(int n, int heads, int hd, int batch) {
  const int splits = (n + ATT_KEYS - 1) / ATT_KEYS;
  return (size_t)batch * heads * splits * (hd + 2);
}

cudaError_t launch_attend(const float *q, long long q_stride, const uint32_t *kv,
                          long long kv_stride, float *part, float *o, long long o_stride, int n,
                          int cols, int heads, int hd, int batch, cudaStream_t s) {
  if (n <= 0 || batch <= 0) return cudaSuccess;
  const int splits = (n + ATT_KEYS - 1) / ATT_KEYS;
  dim3 grid(splits, heads, batch);
  const float scale = 1.0f / sqrtf(float(hd));
  // Plain launches: started early beside the projection before it (a programmatic launch), the
  // many waves of this HBM-bound kernel ran measurably slower (the decoder's cross attention 61 ->
  // 77 us). Both still let the next kernel of the stream launch early.
  attend_kernel<<<grid, ATT_THREADS, 0, s>>>(q, q_stride, kv, kv_stride, part, o, o_stride, n, cols,
                                             hd, scale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  combine_kernel<<<dim3(heads, batch), 64, 0, s>>>(part, o, o_stride, splits, hd);
  return cudaGetLastError();
}

cudaError_t launch_rope(const float *table, void *qkv, int x_f16, long long stride, int rows,
                        int pos, const int *positions, int heads, int hd, int rot, int neox,
                        int sections, cudaStream_t s) {
  const long long total = (long long)rows * sections * heads * (rot / 2);
  if (total <= 0) return cudaSuccess;
  const int half = rot / 2;
  const auto a16 = [](const void *p, unsigned n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
  if (x_f16 && half % 4 == 0 && a16(qkv, 16) && a16(table, 16) && stride % 8 == 0 && hd % 8 == 0) {
    const int per_row = sections * heads * (half / 4);
    const int threads = per_row < 256 ? (per_row + 31) / 32 * 32 : 256;
    const dim3 grid((per_row + threads - 1) / threads, rows < 65535 ? rows : 65535);
    rope4_kernel<<<grid, threads, 0, s>>>(table, reinterpret_cast<__half *>(qkv), stride, rows,
                                          pos, positions, heads, hd, rot, neox, sections);
    return cudaGetLastError();
  }
  long long blocks = (total + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  if (x_f16)
    rope_kernel<__half><<<int(blocks), 256, 0, s>>>(table, reinterpret_cast<__half *>(qkv), stride,
                                                    rows, pos, positions, heads, hd, rot, neox,
                                                    sections);
  else
    rope_kernel<float><<<int(blocks), 256, 0, s>>>(table, reinterpret_cast<float *>(qkv), stride,
                                                   rows, pos, positions, heads, hd, rot, neox,
                                                   sections);
  return cudaGetLastError();
}

cudaError_t launch_gemv(const float *a, long long lda, int wtype, const void *w,
                        const float *scales, const float *bias, float *c, long long ldc, int rows,
                        int n, int k, int epilogue, float alpha, cudaStream_t s) {
  if (rows <= 0 || n <= 0) return cudaSuccess;
  if ((epilogue == kBias || epilogue == kResidual) && k % 32 == 0 && lda % 4 == 0) {
    // Split-K: about two CTAs per SM over the feature groups and k ranges.
    const int groups = (n + GS_F - 1) / GS_F;
    int ks = (2 * 148 + groups - 1) / groups;
    ks = ks < 1 ? 1 : (ks > k / 32 ? k / 32 : ks);
    int kr = (k + ks - 1) / ks;
    kr = (kr + 31) / 32 * 32;
    if (kr > 256) kr = 256;  // 64 KB of W tile
    ks = (k + kr - 1) / kr;
    const size_t smem = size_t(GS_F) * kr * 4;
    if (epilogue == kBias) {
      cudaError_t e = cudaMemset2DAsync(c, size_t(ldc) * 4, 0, size_t(n) * 4, rows, s);
      if (e != cudaSuccess) return e;
    }
    static bool configured[3][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int wi = wtype == 1 ? 0 : wtype == 0 ? 1 : 2;
    if (dev < 64 && !configured[wi][dev]) {
      cudaError_t e = wtype == 1 ? cudaFuncSetAttribute(gemv_split_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536)
                      : wtype == 0 ? cudaFuncSetAttribute(gemv_split_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536)
                                   : cudaFuncSetAttribute(gemv_split_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536);
      if (e != cudaSuccess) return e;
      configured[wi][dev] = true;
    }
    const dim3 grid(groups, ks);
    if (wtype == 1)
      gemv_split_kernel<1><<<grid, 256, smem, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, kr, epilogue, alpha);
    else if (wtype == 0)
      gemv_split_kernel<0><<<grid, 256, smem, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, kr, epilogue, alpha);
    else
      gemv_split_kernel<8><<<grid, 256, smem, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, kr, epilogue, alpha);
    return cudaGetLastError();
  }
  const int grid = (n + 7) / 8;
  if (wtype == 1)
    gemv_kernel<1><<<grid, 256, 0, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, epilogue, alpha);
  else if (wtype == 0)
    gemv_kernel<0><<<grid, 256, 0, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, epilogue, alpha);
  else
    gemv_kernel<8><<<grid, 256, 0, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, epilogue, alpha);
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_gemv_tc_epi(dim3 grid, int ks, size_t smem, cudaStream_t s,
                               const CUtensorMap &map_w, const CUtensorMap &map_a,
                               const float *bias, float *c, long long ldc, int rows, int n, int k,
                               int kr, int stages, int tiles, float alpha, int *err) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, GT_SMEM_MAX);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(GT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = unsigned(ks);
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ks > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gemv_tc_kernel<EPI>, map_w, map_a, bias, c, ldc, rows, n, k, kr,
                            stages, tiles, alpha, err);
}

cudaError_t launch_gemv_tc(const CUtensorMap &map_a, const CUtensorMap &map_w128,
                           const float *bias, float *c, long long ldc, int rows, int n, int k,
                           int epilogue, float alpha, int sms, int *err, cudaStream_t s) {
  if (rows <= 0 || n <= 0) return cudaSuccess;
  if (rows > 32 || k <= 0 || sms <= 0) return cudaErrorInvalidValue;
  // About one CTA per SM. With fewer tiles than SMs, k splits over a cluster of up to 8 CTAs a tile;
  // otherwise each CTA takes every gridDim.x-th tile (at most GT_TMAX) with the whole k.
  const int tiles = (n + GT_N - 1) / GT_N;
  int ks = tiles < sms ? sms / tiles : 1;
  if (ks > GT_MAX_CLUSTER) ks = GT_MAX_CLUSTER;
  if (ks > (k + 63) / 64) ks = (k + 63) / 64;
  if (ks < 1) ks = 1;
  int kr = ((k + ks - 1) / ks + 63) / 64 * 64;
  ks = (k + kr - 1) / kr;
  int grid = ks > 1 ? tiles : (tiles < sms ? tiles : sms);
  if (ks == 1 && grid < (tiles + GT_TMAX - 1) / GT_TMAX) grid = (tiles + GT_TMAX - 1) / GT_TMAX;
  int stages = int((GT_SMEM_MAX - gt_smem_bytes(0)) / GT_W_CHUNK);
  if (stages > GT_MAX_STAGES) stages = GT_MAX_STAGES;
  const size_t smem = gt_smem_bytes(stages);
  const dim3 g(grid, ks);
  switch (epilogue) {
#define WV_GEMV_TC(E) \
  case E:             \
    return launch_gemv_tc_epi<E>(g, ks, smem, s, map_w128, map_a, bias, c, ldc, rows, n, k, kr, \
                                 stages, tiles, alpha, err);
    WV_GEMV_TC(kBias)
    WV_GEMV_TC(kSilu)
    WV_GEMV_TC(kRelu)
    WV_GEMV_TC(kResidual)
    WV_GEMV_TC(kGelu)
    WV_GEMV_TC(kGeluResidual)
    WV_GEMV_TC(kTanh)
#undef WV_GEMV_TC
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace wv
