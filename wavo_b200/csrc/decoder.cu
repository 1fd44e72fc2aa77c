// The Whisper decoder step's ends on the device, so that a greedy decode never leaves the GPU:
//
//   embed_kernel  the token rows of a batch: x[b] = W[token[b]] + positions[pos] + bias, the
//                 reference's `Pass::embed` (src/gpu/mod.rs:1471-1484; CPU `Linear::row` plus the
//                 learned positions, src/cpu/transformer.rs:228-231) with W as the layer stores it
//                 (F32 / BF16 exact in f32, F16 exact, Q8_0 as q·d in f32).
//   pick_cluster_kernel / pick_kernel
//                 the next token of each row from its logits, which the reference computes on the
//                 CPU between steps (src/whisper/search.rs:46-59 `pick`, 76-107 `timestamp_rules`,
//                 111-123 `argmax`): the suppression lists, the timestamp rules over the row's
//                 generated tokens, the first maximum and its log-softmax. A cluster of up to 8
//                 CTAs a row with the row's logits in registers (vocabularies up to 65 536), else
//                 one CTA a row; the logits are edited in place as the reference edits its vector;
//                 f64 sums of exponentials as the reference's.
#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

constexpr int PICK_THREADS = 512;

__global__ void embed_kernel(const void *__restrict__ w, int wtype, const float *__restrict__ d8,
                             const float *__restrict__ bias, const float *__restrict__ positions,
                             const int *__restrict__ tokens, int k, int pos, float *__restrict__ x,
                             long long ldx) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  const int b = int(blockIdx.y);
  const long long t = tokens[b];
  for (int c = int(blockIdx.x * blockDim.x + threadIdx.x); c < k; c += int(gridDim.x * blockDim.x)) {
    float v;
    if (wtype == 0) {
      v = static_cast<const float *>(w)[t * k + c];
    } else if (wtype == 1) {
      v = __half2float(static_cast<const __half *>(w)[t * k + c]);
    } else {
      v = float(static_cast<const int8_t *>(w)[t * k + c]) * d8[(t * k + c) / 32];
    }
    if (positions) v += positions[(long long)pos * k + c];
    x[b * ldx + c] = v + bias[c];
  }
}

// Block-wide reductions (PICK_THREADS threads; `sh` holds a slot per warp).
__device__ __forceinline__ float block_max(float v, float *sh) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = l < PICK_THREADS / 32 ? sh[l] : -INFINITY;
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ double block_sum(double v, double *sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = l < PICK_THREADS / 32 ? sh[l] : 0.0;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The first maximum: the largest value, ties to the lowest index (the reference keeps `best` and
// moves it only on a strictly greater value; with every value -inf it stays at 0).
__device__ __forceinline__ void block_argmax(float &v, int &i, float *shv, int *shi) {
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    shv[w] = v;
    shi[w] = i;
  }
  __syncthreads();
  v = l < PICK_THREADS / 32 ? shv[l] : -INFINITY;
  i = l < PICK_THREADS / 32 ? shi[l] : 0x7fffffff;
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

__global__ void __launch_bounds__(PICK_THREADS)
    pick_kernel(float *__restrict__ logits, long long ld, int vocab, int *__restrict__ history,
                int *__restrict__ hist_len, int max_hist, const int *__restrict__ suppress,
                int n_suppress, const int *__restrict__ begin_suppress, int n_begin, int eot,
                int no_ts, int begin, int max_initial, int *__restrict__ tokens,
                float *__restrict__ logprobs) {
  __shared__ float shf[PICK_THREADS / 32];
  __shared__ int shi[PICK_THREADS / 32];
  __shared__ double shd[PICK_THREADS / 32];
  __shared__ int sh_ts;
  const int b = int(blockIdx.x), tid = int(threadIdx.x);
  // A row whose last pick was EOT is finished: it keeps EOT and adds nothing.
  if (tokens[b] == eot) {
    if (tid == 0 && logprobs) logprobs[b] = 0.0f;
    return;
  }
  float *lg = logits + (long long)b * ld;
  const int *gen = history + (long long)b * max_hist;
  const int n = hist_len[b];
  // Suppression (src/whisper/search.rs:47-54).
  for (int i = tid; i < n_suppress; i += PICK_THREADS)
    if (suppress[i] >= 0 && suppress[i] < vocab) lg[suppress[i]] = -INFINITY;
  if (n == 0)
    for (int i = tid; i < n_begin; i += PICK_THREADS)
      if (begin_suppress[i] >= 0 && begin_suppress[i] < vocab) lg[begin_suppress[i]] = -INFINITY;
  // The timestamp rules (search.rs:76-107): the most recent timestamp among the generated tokens.
  if (tid == 0) {
    int ts = -1;
    for (int i = n - 1; i >= 0; --i)
      if (gen[i] >= begin) {
        ts = gen[i];
        break;
      }
    sh_ts = ts;
  }
  __syncthreads();
  if (tid == 0 && no_ts >= 0 && no_ts < vocab) lg[no_ts] = -INFINITY;
  __syncthreads();
  const bool last = n > 0 && gen[n - 1] >= begin;
  const bool penultimate = n < 2 || gen[n - 2] >= begin;
  const int ts = sh_ts;
  const int low = ts < 0 ? begin : (last && !penultimate ? ts : ts + 1);
  const int init_end = min(begin + max_initial + 1, vocab);
  for (int i = tid; i < vocab; i += PICK_THREADS) {
    bool off = false;
    if (last) off = penultimate ? i >= begin : i < eot;
    if (ts >= 0 && i >= begin && i < low) off = true;
    if (n == 0 && (i < begin || i >= init_end)) off = true;
    if (off) lg[i] = -INFINITY;
  }
  __syncthreads();
  // Timestamps only when their total probability beats every other token.
  float mx = -INFINITY, text = -INFINITY;
  for (int i = tid; i < vocab; i += PICK_THREADS) {
    const float v = lg[i];
    if (i >= begin) mx = fmaxf(mx, v);
    else text = fmaxf(text, v);
  }
  mx = block_max(mx, shf);
  text = block_max(text, shf);
  float mass = -INFINITY;
  if (isfinite(mx)) {
    double s = 0.0;
    for (int i = begin + tid; i < vocab; i += PICK_THREADS) {
      const float v = lg[i];
      if (isfinite(v)) s += exp(double(v - mx));
    }
    s = block_sum(s, shd);
    if (s > 0.0) mass = mx + float(log(s));
  }
  if (mass > text)
    for (int i = tid; i < begin && i < vocab; i += PICK_THREADS) lg[i] = -INFINITY;
  __syncthreads();
  // argmax and its log-softmax (search.rs:111-123).
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  float fm = -INFINITY;
  for (int i = tid; i < vocab; i += PICK_THREADS) {
    const float v = lg[i];
    if (v > bv) {
      bv = v;
      bi = i;
    }
    if (isfinite(v)) fm = fmaxf(fm, v);
  }
  block_argmax(bv, bi, shf, shi);
  const int best = isinf(bv) && bv < 0 ? 0 : bi;
  float lp = 0.0f;
  if (logprobs) {
    fm = block_max(fm, shf);
    double s = 0.0;
    for (int i = tid; i < vocab; i += PICK_THREADS) {
      const float v = lg[i];
      if (isfinite(v)) s += exp(double(v - fm));
    }
    s = block_sum(s, shd);
    lp = lg[best] - (fm + float(log(s)));
  }
  if (tid == 0) {
    tokens[b] = best;
    if (logprobs) logprobs[b] = lp;
    if (best != eot && n < max_hist) {
      history[(long long)b * max_hist + n] = best;
      hist_len[b] = n + 1;
    }
  }
}

// ---- the pick over a cluster: one row on up to 8 CTAs, its logits in registers ----------------
//
// The vocabulary of a row is cut into slices of at most PK_SLICE logits, one CTA a slice (the CTAs
// of a row form a cluster); thread t keeps logits lo + t + 256j of its CTA's slice in registers, so
// that the row is read from memory once and the edited logits are written back only where an edit
// changed them. Three cluster rounds through distributed shared memory: (1) the maxima and first
// maxima of the text part (ids below `begin`) and the timestamp part, over every value and over
// finite values; (2) the f64 sums Σ exp(v - m) over the timestamps' finite values (m their finite
// maximum: the timestamps' mass, and the log-softmax's sum when the text is suppressed) and over
// every finite value (m the finite maximum of the row: the log-softmax's sum otherwise); each
// combined in rank order, so that the result does not depend on timing; (3) the decision, after
// which the CTAs write their edits back and leave together.
constexpr int PK_THREADS = 256;
constexpr int PK_J = 32;                      // logits a thread keeps
constexpr int PK_SLICE = PK_THREADS * PK_J;   // logits a CTA takes
constexpr int PK_MAX_CTAS = 8;

struct PickPart {
  float tx_max, tx_fmax, ts_max, ts_fmax;  // maxima of all values and of finite values
  float tx_bv, ts_bv;                      // first maxima (value, index) of each part
  int tx_bi, ts_bi;
  double s_ts, s_all;                      // round 2 sums
};

__device__ __forceinline__ float ldc_f32(const void *p, uint32_t rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(mapa_shared(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ int ldc_s32(const void *p, uint32_t rank) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(mapa_shared(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ double ldc_f64(const void *p, uint32_t rank) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(mapa_shared(p, rank)) : "memory");
  return v;
}

// (value, index) pairs: the larger value, ties to the lower index.
__device__ __forceinline__ void first_max(float &v, int &i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

__global__ void __launch_bounds__(PK_THREADS)
    pick_cluster_kernel(float *__restrict__ logits, long long ld, int vocab,
                        int *__restrict__ history, int *__restrict__ hist_len, int max_hist,
                        const int *__restrict__ suppress, int n_suppress,
                        const int *__restrict__ begin_suppress, int n_begin, int eot, int no_ts,
                        int begin, int max_initial, int *__restrict__ tokens,
                        float *__restrict__ logprobs, int slice) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  __shared__ uint32_t bits[PK_SLICE / 32];  // the suppression lists' ids in this slice
  __shared__ PickPart part;
  __shared__ float wf[PK_THREADS / 32][6];
  __shared__ int wi[PK_THREADS / 32][2];
  __shared__ double wd[PK_THREADS / 32][2];
  __shared__ int sh_ts;
  __shared__ float g_ts_fmax, g_fm_all;
  __shared__ int g_text_off;
  const int b = int(blockIdx.y), tid = int(threadIdx.x), lane = tid & 31, w = tid >> 5;
  const uint32_t rank = cluster_ctarank();
  const int nct = int(gridDim.x);
  // A row whose last pick was EOT is finished: it keeps EOT and adds nothing (the same decision in
  // every CTA of the row: tokens[b] is written only after the last cluster barrier).
  if (tokens[b] == eot) {
    if (rank == 0 && tid == 0 && logprobs) logprobs[b] = 0.0f;
    return;
  }
  const int lo = int(rank) * slice, hi = min(vocab, lo + slice);
  float *lg = logits + (long long)b * ld;
  const int *gen = history + (long long)b * max_hist;
  const int n = hist_len[b];
  for (int i = tid; i < PK_SLICE / 32; i += PK_THREADS) bits[i] = 0u;
  if (w == 0) {
    // The most recent timestamp among the generated tokens, 32 at a time from the end.
    int ts = -1;
    for (int base = n - 1; base >= 0 && ts < 0; base -= 32) {
      const int i = base - lane;
      const int t = i >= 0 ? gen[i] : -1;
      const unsigned m = __ballot_sync(0xffffffffu, i >= 0 && t >= begin);
      if (m) ts = __shfl_sync(0xffffffffu, t, __ffs(m) - 1);
    }
    if (lane == 0) sh_ts = ts;
  }
  __syncthreads();
  const auto mark = [&](int e) {
    if (e >= lo && e < hi) atomicOr(&bits[(e - lo) >> 5], 1u << ((e - lo) & 31));
  };
  for (int i = tid; i < n_suppress; i += PK_THREADS) mark(suppress[i]);
  if (n == 0)
    for (int i = tid; i < n_begin; i += PK_THREADS) mark(begin_suppress[i]);
  if (tid == 0) mark(no_ts);
  __syncthreads();
  // Suppression and the timestamp rules (search.rs:47-54, 76-107) in registers.
  const bool last = n > 0 && gen[n - 1] >= begin;
  const bool penultimate = n < 2 || gen[n - 2] >= begin;
  const int ts = sh_ts;
  const int low = ts < 0 ? begin : (last && !penultimate ? ts : ts + 1);
  const int init_end = min(begin + max_initial + 1, vocab);
  float v[PK_J];
#pragma unroll
  for (int j = 0; j < PK_J; ++j) {
    const int i = lo + tid + PK_THREADS * j;
    v[j] = i < hi ? lg[i] : -INFINITY;
  }
  uint32_t edited = 0u;
  float tx_max = -INFINITY, tx_f = -INFINITY, ts_max = -INFINITY, ts_f = -INFINITY;
  float tx_bv = -INFINITY, ts_bv = -INFINITY;
  int tx_bi = 0x7fffffff, ts_bi = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < PK_J; ++j) {
    const int i = lo + tid + PK_THREADS * j;
    if (i < hi) {
      bool off = (bits[(i - lo) >> 5] >> ((i - lo) & 31)) & 1u;
      if (last) off = off || (penultimate ? i >= begin : i < eot);
      if (ts >= 0 && i >= begin && i < low) off = true;
      if (n == 0 && (i < begin || i >= init_end)) off = true;
      if (off && v[j] != -INFINITY) {
        v[j] = -INFINITY;
        edited |= 1u << j;
      }
      const float x = v[j];
      if (i >= begin) {
        ts_max = fmaxf(ts_max, x);
        if (isfinite(x)) ts_f = fmaxf(ts_f, x);
        if (x > ts_bv) {
          ts_bv = x;
          ts_bi = i;
        }
      } else {
        tx_max = fmaxf(tx_max, x);
        if (isfinite(x)) tx_f = fmaxf(tx_f, x);
        if (x > tx_bv) {
          tx_bv = x;
          tx_bi = i;
        }
      }
    }
  }
  // Round 1: this CTA's maxima, then the row's.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    tx_max = fmaxf(tx_max, __shfl_xor_sync(0xffffffffu, tx_max, o));
    tx_f = fmaxf(tx_f, __shfl_xor_sync(0xffffffffu, tx_f, o));
    ts_max = fmaxf(ts_max, __shfl_xor_sync(0xffffffffu, ts_max, o));
    ts_f = fmaxf(ts_f, __shfl_xor_sync(0xffffffffu, ts_f, o));
    first_max(tx_bv, tx_bi, __shfl_xor_sync(0xffffffffu, tx_bv, o),
              __shfl_xor_sync(0xffffffffu, tx_bi, o));
    first_max(ts_bv, ts_bi, __shfl_xor_sync(0xffffffffu, ts_bv, o),
              __shfl_xor_sync(0xffffffffu, ts_bi, o));
  }
  if (lane == 0) {
    wf[w][0] = tx_max; wf[w][1] = tx_f; wf[w][2] = ts_max; wf[w][3] = ts_f;
    wf[w][4] = tx_bv; wf[w][5] = ts_bv; wi[w][0] = tx_bi; wi[w][1] = ts_bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int k = 1; k < PK_THREADS / 32; ++k) {
      tx_max = fmaxf(tx_max, wf[k][0]); tx_f = fmaxf(tx_f, wf[k][1]);
      ts_max = fmaxf(ts_max, wf[k][2]); ts_f = fmaxf(ts_f, wf[k][3]);
      first_max(tx_bv, tx_bi, wf[k][4], wi[k][0]);
      first_max(ts_bv, ts_bi, wf[k][5], wi[k][1]);
    }
    part.tx_max = tx_max; part.tx_fmax = tx_f; part.ts_max = ts_max; part.ts_fmax = ts_f;
    part.tx_bv = tx_bv; part.ts_bv = ts_bv; part.tx_bi = tx_bi; part.ts_bi = ts_bi;
  }
  cluster_sync();
  if (tid == 0) {
    for (int p = 0; p < nct; ++p) {
      if (p == int(rank)) continue;
      tx_max = fmaxf(tx_max, ldc_f32(&part.tx_max, p));
      tx_f = fmaxf(tx_f, ldc_f32(&part.tx_fmax, p));
      ts_max = fmaxf(ts_max, ldc_f32(&part.ts_max, p));
      ts_f = fmaxf(ts_f, ldc_f32(&part.ts_fmax, p));
      first_max(tx_bv, tx_bi, ldc_f32(&part.tx_bv, p), ldc_s32(&part.tx_bi, p));
      first_max(ts_bv, ts_bi, ldc_f32(&part.ts_bv, p), ldc_s32(&part.ts_bi, p));
    }
    g_ts_fmax = ts_f;
    g_fm_all = fmaxf(tx_f, ts_f);
  }
  __syncthreads();
  // Round 2: Σ exp(v - m) in f64 over the timestamps' finite values (m their finite maximum) and
  // over every finite value (m the row's finite maximum).
  {
    const float m_ts = g_ts_fmax, m_all = g_fm_all;
    double s_ts = 0.0, s_all = 0.0;
#pragma unroll
    for (int j = 0; j < PK_J; ++j) {
      const int i = lo + tid + PK_THREADS * j;
      if (i < hi && isfinite(v[j])) {
        if (i >= begin) s_ts += exp(double(v[j] - m_ts));
        s_all += exp(double(v[j] - m_all));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s_ts += __shfl_xor_sync(0xffffffffu, s_ts, o);
      s_all += __shfl_xor_sync(0xffffffffu, s_all, o);
    }
    if (lane == 0) {
      wd[w][0] = s_ts;
      wd[w][1] = s_all;
    }
    __syncthreads();
    if (tid == 0) {
      double a = 0.0, c = 0.0;
      for (int k = 0; k < PK_THREADS / 32; ++k) {
        a += wd[k][0];
        c += wd[k][1];
      }
      part.s_ts = a;
      part.s_all = c;
    }
  }
  cluster_sync();
  if (tid == 0) {
    double s_ts = 0.0, s_all = 0.0;
    for (int p = 0; p < nct; ++p) {
      s_ts += p == int(rank) ? part.s_ts : ldc_f64(&part.s_ts, p);
      s_all += p == int(rank) ? part.s_all : ldc_f64(&part.s_all, p);
    }
    // Timestamps only when their total probability beats every other token (search.rs:97-104).
    float mass = -INFINITY;
    if (isfinite(ts_max) && s_ts > 0.0) mass = ts_max + float(log(s_ts));
    const bool text_off = mass > tx_max;
    g_text_off = text_off;
    if (rank == 0) {
      // The first maximum (search.rs:111-123): with every value -inf it stays at 0.
      int best;
      float bv;
      if (text_off) {
        bv = ts_bv;
        best = ts_bi;
      } else {
        bv = tx_bv;
        best = tx_bi;
        first_max(bv, best, ts_bv, ts_bi);
      }
      if (bv == -INFINITY) best = 0;  // every value -inf: logits[0] is -inf too
      if (logprobs) {
        const float fm = text_off ? ts_f : fmaxf(tx_f, ts_f);
        const double s = text_off ? s_ts : s_all;
        logprobs[b] = bv - (fm + float(log(s)));
      }
      tokens[b] = best;
      if (best != eot && n < max_hist) {
        history[(long long)b * max_hist + n] = best;
        hist_len[b] = n + 1;
      }
    }
  }
  __syncthreads();
  // The edits back into the row (the reference edits its vector in place).
  const bool text_off = g_text_off;
#pragma unroll
  for (int j = 0; j < PK_J; ++j) {
    const int i = lo + tid + PK_THREADS * j;
    if (i < hi && (((edited >> j) & 1u) || (text_off && i < begin && v[j] != -INFINITY)))
      lg[i] = -INFINITY;
  }
  cluster_sync();  // every CTA's partials stay until the others have read them
}

}  // namespace

cudaError_t launch_embed(const void *w, int wtype, const float *d8, const float *bias,
                         const float *positions, const int *tokens, int rows, int k, int pos,
                         float *x, long long ldx, cudaStream_t s) {
  if (rows <= 0 || k <= 0) return cudaSuccess;
  const dim3 grid((k + 255) / 256, rows);
  return launch_pdl(embed_kernel, grid, dim3(256), 0, s, w, wtype, d8, bias, positions, tokens, k,
                    pos, x, ldx);
}

cudaError_t launch_pick(float *logits, long long ld, int rows, int vocab, int *history,
                        int *hist_len, int max_hist, const int *suppress, int n_suppress,
                        const int *begin_suppress, int n_begin, int eot, int no_ts, int begin,
                        int max_initial, int *tokens, float *logprobs, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (vocab <= PK_MAX_CTAS * PK_SLICE && rows <= 65535) {
    const int nct = (vocab + PK_SLICE - 1) / PK_SLICE;
    const int slice = (vocab + nct - 1) / nct;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nct, rows);
    cfg.blockDim = dim3(PK_THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(nct);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, pick_cluster_kernel, logits, ld, vocab, history, hist_len,
                              max_hist, suppress, n_suppress, begin_suppress, n_begin, eot, no_ts,
                              begin, max_initial, tokens, logprobs, slice);
  }
  pick_kernel<<<rows, PICK_THREADS, 0, s>>>(logits, ld, vocab, history, hist_len, max_hist,
                                            suppress, n_suppress, begin_suppress, n_begin, eot,
                                            no_ts, begin, max_initial, tokens, logprobs);
  return cudaGetLastError();
}

}  // namespace wv
