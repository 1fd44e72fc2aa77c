// The Whisper decoder step's ends on the device, so that a greedy decode never leaves the GPU:
//
//   embed_kernel  the token rows of a batch: x[b] = W[token[b]] + positions[pos] + bias, the
//                 reference's `Pass::embed` (src/gpu/mod.rs:1471-1484; CPU `Linear::row` plus the
//                 learned positions, src/cpu/transformer.rs:228-231) with W as the layer stores it
//                 (F32 / BF16 exact in f32, F16 exact, Q8_0 as q·d in f32).
//   pick_kernel   the next token of each row from its logits, which the reference computes on the
//                 CPU between steps (src/whisper/search.rs:46-59 `pick`, 76-107 `timestamp_rules`,
//                 111-123 `argmax`): the suppression lists, the timestamp rules over the row's
//                 generated tokens, the first maximum and its log-softmax. One CTA a row; the
//                 logits are edited in place as the reference edits its vector; f64 sums of
//                 exponentials as the reference's.
#include "kernels.cuh"

namespace wv {
namespace {

constexpr int PICK_THREADS = 512;

__global__ void embed_kernel(const void *__restrict__ w, int wtype, const float *__restrict__ d8,
                             const float *__restrict__ bias, const float *__restrict__ positions,
                             const int *__restrict__ tokens, int k, int pos, float *__restrict__ x,
                             long long ldx) {
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

}  // namespace

cudaError_t launch_embed(const void *w, int wtype, const float *d8, const float *bias,
                         const float *positions, const int *tokens, int rows, int k, int pos,
                         float *x, long long ldx, cudaStream_t s) {
  if (rows <= 0 || k <= 0) return cudaSuccess;
  const dim3 grid((k + 255) / 256, rows);
  embed_kernel<<<grid, 256, 0, s>>>(w, wtype, d8, bias, positions, tokens, k, pos, x, ldx);
  return cudaGetLastError();
}

cudaError_t launch_pick(float *logits, long long ld, int rows, int vocab, int *history,
                        int *hist_len, int max_hist, const int *suppress, int n_suppress,
                        const int *begin_suppress, int n_begin, int eot, int no_ts, int begin,
                        int max_initial, int *tokens, float *logprobs, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  pick_kernel<<<rows, PICK_THREADS, 0, s>>>(logits, ld, vocab, history, hist_len, max_hist,
                                            suppress, n_suppress, begin_suppress, n_begin, eot,
                                            no_ts, begin, max_initial, tokens, logprobs);
  return cudaGetLastError();
}

}  // namespace wv
