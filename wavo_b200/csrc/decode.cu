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
__global__ void __launch_bounds__(ATT_THREADS)
    attend_kernel(const float *__restrict__ q, long long q_stride, const uint32_t *__restrict__ kv,
                  long long kv_stride, float *__restrict__ part, float *__restrict__ o,
                  long long o_stride, int n, int cols, int hd, float scale) {
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
  if (jt < nk) {
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

}  // namespace

cudaError_t launch_pack_cache(const float *x, long long src, long long stride, uint32_t *cache,
                              int rows, int d, int cols, int col, long long x_batch,
                              long long cache_batch, int batch, cudaStream_t s) {
  const long long total = (long long)rows * d;
  if (total <= 0 || batch <= 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  pack_cache_kernel<<<dim3(int(blocks), batch), 256, 0, s>>>(x, src, stride, cache, rows, d, cols,
                                                             col, x_batch, cache_batch);
  return cudaGetLastError();
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
  const int grid = (n + 7) / 8;
  if (wtype == 1)
    gemv_kernel<1><<<grid, 256, 0, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, epilogue, alpha);
  else if (wtype == 0)
    gemv_kernel<0><<<grid, 256, 0, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, epilogue, alpha);
  else
    gemv_kernel<8><<<grid, 256, 0, s>>>(a, lda, w, scales, bias, c, ldc, rows, n, k, epilogue, alpha);
  return cudaGetLastError();
}

}  // namespace wv
