/*
 * wavo_cuda.h — C ABI of the wavo-b200 attention path (libwavo_cuda.so / libwavo_cuda.a, sm_100a).
 *
 * This is the drop-in boundary for the multi-head attention path of vladkens/wavo: the encoders'
 * self-attention (Parakeet relative positions, GigaAM rotary, Whisper) with their QKV / output /
 * linear_pos projections, and the Whisper decoder's attention over F16 KV caches. Each entry point
 * replaces one method of the reference's GPU backend op interface (`gpu::Gpu` / `gpu::Pass`,
 * src/gpu/mod.rs), cited beside it; the argument meanings and buffer layouts are the reference's.
 *
 * Conventions
 *  - Pointers named as buffers are device pointers (cudaMalloc or wavo_malloc), except where a
 *    comment says "host".
 *  - Calls enqueue work on the context's stream and return at once; argument errors return at
 *    once; device faults and kernel wait timeouts surface at wavo_sync (as the reference's surface
 *    at `Gpu::run` / `Gpu::finish`, src/gpu/mod.rs:969-1003).
 *  - No exception crosses this boundary. A context serialises its calls with an internal mutex
 *    (the reference's `Gpu::busy`, src/gpu/mod.rs:233-235); wavo_linear_create may be called from
 *    many threads at once.
 *  - Element types: WAVO_F32 is the reference's buffer type; WAVO_F16 is the B200 fast path (the
 *    GEMM writes f16 operands the attention kernel loads with TMA, and the attention writes f16
 *    rows the output projection loads directly).
 */
#ifndef WAVO_CUDA_H
#define WAVO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum wavo_status {
  WAVO_OK = 0,
  WAVO_EINVAL = 1,       /* bad argument: shape, layout, type (reference: Error::Model via bail!) */
  WAVO_ENOMEM = 2,       /* device allocation failed */
  WAVO_ECUDA = 3,        /* CUDA runtime error (reference: Error::Gpu) */
  WAVO_ETIMEDOUT = 4,    /* wavo_sync ran past its limit (reference: Error::Poll) */
  WAVO_EUNSUPPORTED = 5, /* no sm_100 device, or a shape outside the kernels' range */
  WAVO_EDEVICE = 6       /* a kernel's bounded wait gave up (the device error word was set) */
} wavo_status;

typedef enum wavo_dtype { WAVO_F32 = 0, WAVO_F16 = 1 } wavo_dtype;

/* GGUF tensor types: the three the reference reads (src/gguf.rs:14-38), and BF16 (GGUF id 30),
 * which the reference does not read; BF16 weights are converted to the GEMM's f16 at load. */
typedef enum wavo_ggml_type {
  WAVO_GGML_F32 = 0,
  WAVO_GGML_F16 = 1,
  WAVO_GGML_Q8_0 = 8,
  WAVO_GGML_BF16 = 30
} wavo_ggml_type;

/* The reference's `Epilogue` (src/gpu/mod.rs:431-456), in its kernel order. */
typedef enum wavo_epilogue {
  WAVO_EPI_BIAS = 0,
  WAVO_EPI_SILU = 1,
  WAVO_EPI_RELU = 2,
  WAVO_EPI_RESIDUAL = 3, /* c += alpha * (a·W^T + b) */
  WAVO_EPI_GELU = 4,
  WAVO_EPI_GELU_RESIDUAL = 5,
  WAVO_EPI_TANH = 6
} wavo_epilogue;

typedef struct wavo_ctx wavo_ctx;
typedef struct wavo_linear wavo_linear;
typedef struct wavo_gguf wavo_gguf;
typedef struct wavo_graph wavo_graph;

/* ---- device and context: replaces Gpu::new (src/gpu/mod.rs:461-578) -------------------- */

/* Number of CUDA devices visible to this process. */
int wavo_device_count(void);

/* A context on `device`: checks the device is sm_100 (B200 class), creates a stream and the
 * device error word. Replaces Gpu::new (src/gpu/mod.rs:461-578). */
wavo_status wavo_create(int device, wavo_ctx **out);
void wavo_destroy(wavo_ctx *ctx);

/* The last error message of the context. With ctx NULL: the last error of a call without a
 * context (wavo_create, wavo_attend_batch_noalloc) made by the calling thread; each thread has
 * its own, valid until that thread's next such call fails. */
const char *wavo_last_error(const wavo_ctx *ctx);

/* Runs the context's work on `stream` (a cudaStream_t; NULL is the CUDA default stream). A new
 * context runs on a stream of its own, which wavo_own_stream returns. */
wavo_status wavo_set_stream(wavo_ctx *ctx, void *stream);
void *wavo_get_stream(const wavo_ctx *ctx);
void *wavo_own_stream(const wavo_ctx *ctx);
int wavo_sm_count(const wavo_ctx *ctx);

/* ---- buffers: replaces Gpu::buffer / upload / write / readback (src/gpu/mod.rs:741-756) -- */

wavo_status wavo_malloc(wavo_ctx *ctx, size_t bytes, void **out);
wavo_status wavo_free(wavo_ctx *ctx, void *ptr);
/* Host -> device and device -> host copies on the context's stream (host: pinned for overlap). */
wavo_status wavo_upload(wavo_ctx *ctx, void *dst, const void *host_src, size_t bytes);
wavo_status wavo_download(wavo_ctx *ctx, void *host_dst, const void *src, size_t bytes);
wavo_status wavo_memset(wavo_ctx *ctx, void *dst, int value, size_t bytes);
/* Grows the context's scratch so that the calls that follow allocate nothing (needed before a
 * graph capture). */
wavo_status wavo_reserve(wavo_ctx *ctx, size_t workspace_bytes);
/* Waits for the context's stream, at most timeout_ms (0: no limit). Device faults, the kernels'
 * wait timeouts (WAVO_EDEVICE) and the limit (WAVO_ETIMEDOUT) surface here. Replaces the
 * completion check of Gpu::run / Gpu::finish (src/gpu/mod.rs:969-1003). */
wavo_status wavo_sync(wavo_ctx *ctx, uint32_t timeout_ms);

/* ---- linear layers: replaces Gpu::linear (src/gpu/mod.rs:758-834) ------------------------ */

/* Weights [rows][k] as GGUF tensor bytes of `ggml_type` (host), stacked along the rows, and a host
 * bias: NULL/0 for zeros, `rows` values, or rows + dual values — the extra `dual` values write the
 * first `dual` outputs a second time after the others with those biases (one q with the two
 * position biases u and v, src/conformer.rs:174-200). k % 32 == 0. Output columns: the rows when
 * a multiple of 32, else the rows padded to 64 (those outputs are epilogue(0)), plus `dual`.
 * Thread-safe. */
wavo_status wavo_linear_create(wavo_ctx *ctx, int ggml_type, uint32_t rows, uint32_t k,
                               const void *data, const float *bias, size_t bias_len,
                               wavo_linear **out);
void wavo_linear_destroy(wavo_linear *l);
/* Linear::width (src/gpu/mod.rs:408-413): output columns including the dual ones. */
uint32_t wavo_linear_width(const wavo_linear *l);
uint32_t wavo_linear_k(const wavo_linear *l);

/* ---- the log-mel frontend: replaces parakeet::frontend::Frontend (src/parakeet/frontend.rs) ---
 * 16 kHz pcm (device f32) to 128 log-mel bins a 10 ms frame, time-major: pre-emphasis, Hann(400)
 * in an FFT of 512 (f64, the reference's operations in its order), power to f32, the Slaney
 * filterbank, ln(mel + 2^-24). The first frontend call on a context makes its tables (a device
 * allocation): make it before any stream capture. */

/* Frontend::log_mel (src/parakeet/frontend.rs:74-108): frames f0 .. f1 of the whole pcm
 * (f1 <= samples / 160 + 1), each computed from only the samples it covers, into mel
 * [f1 - f0][128]. */
wavo_status wavo_log_mel(wavo_ctx *ctx, const float *pcm, uint64_t samples, uint64_t f0,
                         uint64_t f1, float *mel);
/* Frontend::compute (src/parakeet/frontend.rs:50-70): all samples / 160 + 1 frames, each mel bin
 * normalised over all frames but the last (unbiased, + 1e-5), the last frame zero; *frames gets
 * the count, 0 (and nothing written) below 3 frames. mel holds samples / 160 + 1 rows of 128. */
wavo_status wavo_mel_features(wavo_ctx *ctx, const float *pcm, uint64_t samples, float *mel,
                              uint64_t *frames);

/* Parakeet's 8x conv subsampling (src/parakeet/cpu.rs:60-174, GPU src/parakeet/encoder.rs:103-121):
 * from mel [frames][128] (of which `valid` are audio, the rest padding), conv0 (3x3, stride 2, 1 ->
 * ch) + ReLU, conv2 (depthwise 3x3, stride 2) with its rows from half(half(valid)) on zero, conv3
 * (pointwise, the linear layer ch -> ch) + ReLU, conv5 (depthwise), conv6 (pointwise) + ReLU,
 * [t][16][ch] to [t][ch·16], and the output projection `out` (16·ch -> d) + bias into x [t][d],
 * t = half(half(half(frames - 1))) with half(n) = (n - 1) / 2 + 1 (*t_out gets it). Taps are
 * device f32 [9][ch] (time tap, then frequency tap), biases [ch]; ch % 32 == 0. The intermediate
 * images go to `scratch` (device, 256-byte aligned, wavo_subsample_scratch_bytes of them). */
uint64_t wavo_subsample_scratch_bytes(uint32_t frames, uint32_t ch);
wavo_status wavo_subsample(wavo_ctx *ctx, const float *mel, uint32_t frames, uint32_t valid,
                           uint32_t ch, const float *w0, const float *b0, const float *w2,
                           const float *b2, const wavo_linear *conv3, const float *w5,
                           const float *b5, const wavo_linear *conv6, const wavo_linear *out,
                           float *x, void *scratch, uint32_t *t_out);

/* wavo_subsample over n segments in one call (the reference subsamples each piece on its own,
 * src/parakeet/cpu.rs:60-174 per piece; each segment's rows here equal that call's): segment s's
 * frames[s] mel rows (valid[s] of them audio) follow segment s - 1's in `mel`, and its t_s output
 * rows follow segment s - 1's in x (t_out[s] gets t_s when t_out is not NULL). conv0/conv2, conv3
 * and conv5 run segment by segment; conv6, the flatten and the output projection once over every
 * segment's rows. scratch: wavo_subsample_batch_scratch_bytes of device memory, 256-byte aligned. */
uint64_t wavo_subsample_batch_scratch_bytes(const uint32_t *frames, uint32_t n, uint32_t ch);
wavo_status wavo_subsample_batch(wavo_ctx *ctx, const float *mel, const uint32_t *frames,
                                 const uint32_t *valid, uint32_t n, uint32_t ch, const float *w0,
                                 const float *b0, const float *w2, const float *b2,
                                 const wavo_linear *conv3, const float *w5, const float *b5,
                                 const wavo_linear *conv6, const wavo_linear *out, float *x,
                                 void *scratch, uint32_t *t_out);

/* ---- GGUF files: replaces gguf::Gguf / gguf::Tensor (src/gguf.rs) ----------------------------
 * Host calls without a context: errors read from wavo_last_error(NULL). A wavo_gguf may be read
 * from many threads at once. */

/* Gguf::open (src/gguf.rs:122-128): reads and checks the header (GGUF v3; tensors F32, F16 or Q8_0,
 * inside the file); tensor data is read when used. */
wavo_status wavo_gguf_open(const char *path, wavo_gguf **out);
void wavo_gguf_close(wavo_gguf *g);
/* The tensors in file order. */
uint32_t wavo_gguf_tensor_count(const wavo_gguf *g);
const char *wavo_gguf_tensor_name(const wavo_gguf *g, uint32_t i);
/* Gguf::tensor (src/gguf.rs:241-249): the tensor `name`, which must have exactly the ggml-order
 * dims (dims[0] contiguous; NULL skips the check); its GGUF type and data bytes. */
wavo_status wavo_gguf_tensor(const wavo_gguf *g, const char *name, const uint64_t *dims,
                             uint32_t n_dims, int *ggml_type, uint64_t *bytes);
/* The tensor's dims (up to cap of them written); returns how many it has, 0 if there is none. */
uint32_t wavo_gguf_tensor_dims(const wavo_gguf *g, const char *name, uint64_t *dims, uint32_t cap);
/* Tensor::read (src/gguf.rs:258-272): `bytes` of the tensor's data from byte `offset` (host). */
wavo_status wavo_gguf_read(const wavo_gguf *g, const char *name, uint64_t offset, void *dst,
                           uint64_t bytes);
/* Metadata (src/gguf.rs:190-240 `get` / `optional` / `array`): has (1/0); an integer of any GGUF
 * integer type; an f32/f64; a bool; a UTF-8 string (a pointer into the header, not
 * NUL-terminated, valid until close); an array's item type and length; and all items of an array
 * as integers, floats or strings (a NULL output for a kind the array does not hold). */
int wavo_gguf_has(const wavo_gguf *g, const char *key);
wavo_status wavo_gguf_get_int(const wavo_gguf *g, const char *key, int64_t *v);
wavo_status wavo_gguf_get_float(const wavo_gguf *g, const char *key, double *v);
wavo_status wavo_gguf_get_bool(const wavo_gguf *g, const char *key, int *v);
wavo_status wavo_gguf_get_str(const wavo_gguf *g, const char *key, const char **s, uint64_t *len);
wavo_status wavo_gguf_array(const wavo_gguf *g, const char *key, uint32_t *item_type,
                            uint64_t *len);
wavo_status wavo_gguf_array_items(const wavo_gguf *g, const char *key, int64_t *ints,
                                  double *floats, const char **strs, uint64_t *lens,
                                  uint64_t cap);

/* Gpu::linear over GGUF tensors (src/gpu/mod.rs:758-827 `upload_linear`): the tensors `names`
 * (same type and k = elements / last dim, k % 32 == 0) stacked by rows, with a bias as in
 * wavo_linear_create. The tensors' bytes are streamed from the file to the device in pinned
 * pieces and turned into the device forms there (Q8_0 blocks into the int8 values, scales and f16
 * copy that the GEMM, its Q8_0 prologue and the gemv read through TMA): the same layer as
 * wavo_linear_create on the same bytes. Waits for the upload; serialised with the context's
 * other calls. */
wavo_status wavo_linear_from_gguf(wavo_ctx *ctx, const wavo_gguf *g, const char *const *names,
                                  uint32_t count, const float *bias, size_t bias_len,
                                  wavo_linear **out);

/* ---- projections: replaces Pass::gemm (src/gpu/mod.rs:1394-1425) and Pass::gemv (1461-1467) */

/* c = epilogue(a·W^T + b) for m rows of a ([m][lda], a_dtype) into c ([m][ldc], c_dtype); lda = 0
 * means k, ldc = 0 means wavo_linear_width. a and W are rounded to f16 (the reference GPU GEMM's
 * rounding); sums in f32. */
wavo_status wavo_gemm(wavo_ctx *ctx, const void *a, int a_dtype, uint32_t lda, const wavo_linear *l,
                      void *c, int c_dtype, uint32_t ldc, uint32_t m, int epilogue, float alpha);

/* How wavo_gemm reads a Q8_0 layer's weights. The reference's GEMM dequantises Q8_0 blocks as it
 * stages each K-step (src/gpu/gemm.wgsl:105-130); WAVO_Q8_PROLOGUE does the same (int8 values and
 * scales by TMA, converted to f16 tiles in shared memory: one byte a weight from HBM), while
 * WAVO_Q8_DEQUANT reads the f16 copy made at wavo_linear_create. Both give bit-identical results.
 * WAVO_Q8_AUTO (the default) is the faster of the two at every measured shape, the f16 copy: the
 * converters' shared-memory traffic costs more than the halved weight bytes save (the weights are
 * L2-resident across row tiles). Returns the previous mode. */
enum { WAVO_Q8_AUTO = 0, WAVO_Q8_DEQUANT = 1, WAVO_Q8_PROLOGUE = 2 };
int wavo_set_q8_gemm(wavo_ctx *ctx, int mode);

/* Pass::gemv: c[offset..] = epilogue(a·W^T + b) for one f32 row, W not rounded (f32 sums). */
wavo_status wavo_gemv(wavo_ctx *ctx, const float *a, const wavo_linear *l, float *c, int epilogue,
                      float alpha, uint32_t offset);
/* The same for `rows` rows at once (the decoder of a batch of segments): a [rows][lda],
 * c [rows][ldc]. rows <= 32. */
wavo_status wavo_gemv_rows(wavo_ctx *ctx, const float *a, uint32_t lda, const wavo_linear *l,
                           float *c, uint32_t ldc, uint32_t rows, int epilogue, float alpha);

/* ---- encoder attention: replaces Pass::attention (src/gpu/mod.rs:1556-1605) --------------- */

/* Pass::attention over one segment of t rows, in the reference's three layouts:
 *   v != NULL, pos == NULL : qk [t][q | k] and v [t][heads·hd]  (rotary: GigaAM)
 *   v == NULL, pos == NULL : qk [t][q | k | v]                   (Whisper)
 *   v == NULL, pos != NULL : qk [t][q+u | k | v | q+v] and pos [pos_rows(t)][heads·hd], row r the
 *                            projected relative position t + 15 - r (Parakeet): score (i, j) =
 *                            ((q+u)_i·k_j + (q+v)_i·pos[j - i + t + 15]) / sqrt(hd).
 * o [t][heads·hd]. `dtype` is the element type of qk, v, pos and o. hd <= 128. */
wavo_status wavo_attention(wavo_ctx *ctx, const void *qk, const void *v, const void *pos, void *o,
                           uint32_t t, uint32_t heads, uint32_t hd, int dtype);

/* The same over `nseg` independent segments in one launch (the reference runs one at a time,
 * src/lib.rs:844-900): the operands hold `rows` rows, segment z is rows seg_start[z] ..
 * + seg_len[z] of every operand (seg_start, seg_len: device int32 arrays); max_len >= every
 * seg_len. A key-padding mask is the same call with the padded rows left out of seg_len. With
 * positions, pos holds pos_rows(pos_t) rows, row r the relative position pos_t + 15 - r,
 * pos_t >= every seg_len, and serves all segments. o has o_dtype; its rows outside the segments
 * are left as they are. */
wavo_status wavo_attention_varlen(wavo_ctx *ctx, const void *qk, const void *v, const void *pos,
                                  void *o, uint32_t rows, const int32_t *seg_start,
                                  const int32_t *seg_len, uint32_t nseg, uint32_t max_len,
                                  uint32_t pos_t, uint32_t heads, uint32_t hd, int dtype,
                                  int o_dtype);

/* wavo_attention_varlen over f16 rows [q | k | v] with rotary positions on q and k applied inside
 * the attention kernel: the reference rotates the rows first (Pass::rope, src/gpu/mod.rs:1630-1649,
 * then Pass::attention); here each Q tile and K block is rotated as the kernel stages it, and the
 * rows in memory are left as they are. Row i of a segment takes table row pos + i (rot / 2 cosines,
 * then as many sines; table_rows >= pos + max_len); NEOX pairs (i, i + rot/2) or adjacent pairs
 * (2i, 2i + 1), as wavo_rope. Needs 16-byte aligned rows, heads of 16, 32, 48, 64 or 128, rot / 2
 * (neox) or rot a multiple of 8; other shapes return WAVO_EUNSUPPORTED (use wavo_rope_rows, then
 * wavo_attention_varlen). */
wavo_status wavo_attention_rope_varlen(wavo_ctx *ctx, const void *qkv, void *o, uint32_t rows,
                                       const int32_t *seg_start, const int32_t *seg_len,
                                       uint32_t nseg, uint32_t max_len, uint32_t heads,
                                       uint32_t hd, const float *table, uint32_t table_rows,
                                       uint32_t pos, uint32_t rot, int neox, int o_dtype);

/* ---- the rest of the encoder block around the attention ----------------------------------- */

/* Pass::layer_norm (src/gpu/mod.rs:1431-1449; CPU src/cpu/ops.rs:65-110): per row of f32 x
 * [rows][cols], y = (x - mean)·rstd·w + b with rstd = 1/sqrt(variance + 1e-5), into y (y_dtype).
 * With a table (NULL: none), yr (y_dtype) gets y with NEOX rotary pairs (i, i + hd/2) rotated inside
 * each head of hd: table row positions[r] (device int32; NULL: r) of hd/2 cosines, then hd/2 sines
 * (GigaAM's rotary input to its Q/K projection). cols <= 2048. */
wavo_status wavo_layer_norm(wavo_ctx *ctx, const float *x, const float *w, const float *b, void *y,
                            int y_dtype, uint32_t rows, uint32_t cols, const float *table,
                            const int32_t *positions, void *yr, uint32_t hd);

/* Pass::conv_glu (src/gpu/mod.rs:1538-1566; CPU src/cpu/ops.rs:133-182): the Conformer conv module
 * between its pointwise convs. From h [t][2·ch] (f32, left as it is): GLU (first half ·
 * sigmoid(second half)), the depthwise conv over frames (odd kernel <= 63, centred; dw_w
 * [ch][kernel] as the GGUF tensor stores it, dw_b [ch]), then LayerNorm over the channels
 * (WAVO_CONV_LAYER_NORM: n_w, n_b as its weight and bias) or the per-channel affine n_w·x + n_b
 * (WAVO_CONV_AFFINE, a folded batch norm), then SiLU, into y [t][ch] (y_dtype). */
enum { WAVO_CONV_LAYER_NORM = 0, WAVO_CONV_AFFINE = 1 };
wavo_status wavo_conv_glu(wavo_ctx *ctx, const float *h, const float *dw_w, const float *dw_b,
                          uint32_t kernel, const float *n_w, const float *n_b, int norm, void *y,
                          int y_dtype, uint32_t t, uint32_t ch);
/* The same over nseg independent segments packed in `rows` rows (device int32 seg_start, seg_len;
 * max_len >= every seg_len): the conv does not reach across a segment's ends. Rows of y outside
 * every segment are overwritten with unspecified values. */
wavo_status wavo_conv_glu_varlen(wavo_ctx *ctx, const float *h, const float *dw_w,
                                 const float *dw_b, uint32_t kernel, const float *n_w,
                                 const float *n_b, int norm, void *y, int y_dtype, uint32_t rows,
                                 const int32_t *seg_start, const int32_t *seg_len, uint32_t nseg,
                                 uint32_t max_len, uint32_t ch);

/* ---- the decoder step's ends: a greedy decode that stays on the device ----------------------- */

/* Pass::embed (src/gpu/mod.rs:1471-1484) for a batch: x[b] (f32, row stride ldx; 0 means k) =
 * row tokens[b] of the layer's weights (device int32 token ids) + row `pos` of the f32 positions
 * table [.][k] (NULL: none) + the layer's bias. The weights as stored: F32/BF16 and F16 exact, Q8_0
 * as q·d. */
wavo_status wavo_embed_rows(wavo_ctx *ctx, const wavo_linear *l, const float *positions,
                            const int32_t *tokens, uint32_t rows, uint32_t pos, float *x,
                            uint32_t ldx);

/* The next token of each of `rows` rows, on the device (no reference counterpart on the GPU: the
 * reference picks on the CPU between steps, src/whisper/search.rs:46-59, 76-107, 111-123): per row
 * b, logits[b] (f32 [vocab], row stride ld; edited in place as the reference edits its vector) get
 * the suppression lists (suppress; begin_suppress while the row has generated nothing), the
 * timestamp rules over the row's generated tokens history[b][0 .. hist_len[b]) (no
 * <|notimestamps|>; timestamps in pairs, never decreasing; the first token a timestamp of at most
 * max_initial steps; timestamps only when their total probability beats every other token), then
 * the first maximum. tokens[b] gets it (and logprobs[b], if non-NULL, its log-softmax), and it is
 * appended to the row's history unless it is EOT. A row whose tokens[b] is EOT on entry is
 * finished and stays so. Token ids: `eot`, `no_timestamps`, and timestamps from `begin`. */
wavo_status wavo_pick(wavo_ctx *ctx, float *logits, uint32_t ld, uint32_t rows, uint32_t vocab,
                      int32_t *history, int32_t *hist_len, uint32_t max_hist,
                      const int32_t *suppress, uint32_t n_suppress,
                      const int32_t *begin_suppress, uint32_t n_begin, uint32_t eot,
                      uint32_t no_timestamps, uint32_t begin, uint32_t max_initial,
                      int32_t *tokens, float *logprobs);

/* pos_rows (src/gpu/mod.rs:1060-1065): 2t + 15. */
uint32_t wavo_pos_rows(uint32_t t);

/* Pass::rope (src/gpu/mod.rs:1630-1649): in place over rows [q | k | v] of heads x hd at positions
 * pos..: in q's and k's heads the pairs (2i, 2i+1) for 2i < rot rotate, or with neox (i, i+rot/2);
 * the table holds per position rot/2 cosines, then as many sines. `stride` = 0 means 3·heads·hd. */
wavo_status wavo_rope(wavo_ctx *ctx, const float *table, void *qkv, int dtype, uint32_t stride,
                      uint32_t rows, uint32_t pos, uint32_t heads, uint32_t hd, uint32_t rot,
                      int neox);

/* wavo_rope with the table row of each row given (device int32 `positions`, e.g. the position of
 * each row inside its own segment when segments are packed one after another); NULL means
 * pos + row, as wavo_rope. */
wavo_status wavo_rope_rows(wavo_ctx *ctx, const float *table, void *qkv, int dtype,
                           uint32_t stride, uint32_t rows, uint32_t pos, const int32_t *positions,
                           uint32_t heads, uint32_t hd, uint32_t rot, int neox);

/* ---- decoder attention: replaces Pass::pack (src/gpu/mod.rs:1507-1522), Pass::attend
 * (1485-1505) and attend_len (1053-1059) -------------------------------------------------- */

/* Pass::pack: rows rows of x (f32) from float src on, stride floats apart, each K then V of d
 * floats, into the F16 cache (32-bit words) of cols positions at positions col..: K transposed
 * (pair i of position j at word i·cols + j), then V by position (word d/2·cols + j·d/2 + i). */
wavo_status wavo_pack(wavo_ctx *ctx, const float *x, uint32_t src, uint32_t stride, void *cache,
                      uint32_t rows, uint32_t d, uint32_t cols, uint32_t col);

/* wavo_pack for `batch` segments in one launch: segment b reads x + b·x_batch floats and writes
 * the cache at cache + b·cache_batch 32-bit words (the decoder of a batch of segments). */
wavo_status wavo_pack_batch(wavo_ctx *ctx, const float *x, uint32_t src, uint32_t stride,
                            uint64_t x_batch, void *cache, uint64_t cache_batch, uint32_t rows,
                            uint32_t d, uint32_t cols, uint32_t col, uint32_t batch);

/* attend_len: floats of wavo_attend's `part` scratch for up to n keys (per segment). */
size_t wavo_attend_len(uint32_t n, uint32_t heads, uint32_t hd);

/* Pass::attend: one query per head, q [heads·hd] (rounded to f16), over keys 0..n of a cache of
 * cols positions (see wavo_pack), into o [heads·hd], through part (wavo_attend_len floats). */
wavo_status wavo_attend(wavo_ctx *ctx, const float *q, const void *kv, float *part, float *o,
                        uint32_t n, uint32_t cols, uint32_t heads, uint32_t hd);

/* The same for `batch` segments in one launch: segment b's query at q + b·q_stride floats, its
 * cache at kv + b·kv_stride 32-bit words, its output at o + b·o_stride floats; part holds
 * batch·wavo_attend_len(n, heads, hd) floats. */
wavo_status wavo_attend_batch(wavo_ctx *ctx, const float *q, uint64_t q_stride, const void *kv,
                              uint64_t kv_stride, float *part, float *o, uint64_t o_stride,
                              uint32_t n, uint32_t cols, uint32_t heads, uint32_t hd,
                              uint32_t batch);

/* Most floats of split scratch wavo_attend_batch_noalloc can use (1 MiB): enough for
 * batch·heads·ceil(n/1024)·(hd+2) ≤ 262144, e.g. 99 Whisper-large segments × 20 heads over the
 * 1500 encoder frames with heads of 64. */
#define WAVO_ATTEND_NOALLOC_PART_FLOATS (1u << 18)

/* wavo_attend_batch with no context and no caller scratch: the split partials live in a fixed
 * device array inside the library (WAVO_ATTEND_NOALLOC_PART_FLOATS floats per device), and the
 * launch goes to `stream` (a cudaStream_t; NULL = the default stream) on the calling thread's
 * current device. No reference counterpart (the reference's Pass::attend, src/gpu/mod.rs:1485-1505,
 * takes its `part` buffer from the caller). For callers that cannot allocate device memory at the
 * call: a host that owns every device allocation itself, code recording a stream capture (no
 * cudaMalloc there), a decode loop in which an allocation would synchronise the device.
 * - Allocates nothing: no cudaMalloc / cudaFree, no context. The first call on each device does a
 *   one-time set-up (it looks the array up, which may load the library's device code), so make it
 *   before any stream capture that includes this call.
 * - Calls that overlap on the GPU (on different streams, or from different threads without
 *   ordering) share the array and race: order them on one stream or with events.
 * - Nothing needs zeroing: every partial the combine step reads is written first in the same call.
 * - Returns WAVO_EINVAL, with wavo_last_error(NULL) saying why, when the partials would exceed
 *   WAVO_ATTEND_NOALLOC_PART_FLOATS (split the batch), and for the argument errors of
 *   wavo_attend_batch. */
wavo_status wavo_attend_batch_noalloc(const float *q, uint64_t q_stride, const void *kv,
                                      uint64_t kv_stride, float *o, uint64_t o_stride, uint32_t n,
                                      uint32_t cols, uint32_t heads, uint32_t hd, uint32_t batch,
                                      void *stream);

/* ---- graphs: record a sequence of calls once, replay it with one launch ----------------- */

/* Starts capturing the context's stream (the context's own stream must be current; reserve the
 * scratch first). Every call until wavo_capture_end is recorded, not run. */
wavo_status wavo_capture_begin(wavo_ctx *ctx);
wavo_status wavo_capture_end(wavo_ctx *ctx, wavo_graph **out);
wavo_status wavo_graph_launch(wavo_ctx *ctx, const wavo_graph *g);
void wavo_graph_destroy(wavo_graph *g);

/* ---- self-checks of the device building blocks (no reference counterpart) -------------- */

/* Test support for the completion check (Gpu::run, src/gpu/mod.rs:969-1003): enqueues one warp
 * that waits on an mbarrier nothing arms, through the same bounded wait every kernel of this
 * library uses, with a limit of `limit_cycles` SM cycles (1 .. the kernels' ~1 s default). The
 * wait gives up, the kernel returns, and the next wavo_sync reports WAVO_EDEVICE; the context
 * stays usable. */
wavo_status wavo_selftest_wait_timeout(wavo_ctx *ctx, uint64_t limit_cycles);

/* y[i] = 2^x[i] (device buffers of n floats) by the FMA-pipe polynomial the attention softmax
 * computes part of its exponentials with, for x in [-125, 8] (below -125 it returns 2^-125). */
wavo_status wavo_selftest_exp2(wavo_ctx *ctx, const float *x, float *y, uint32_t n);

/* ---- sharding: the segment partition of the multi-GPU runner ---------------------------- */

/* Longest-processing-time-first assignment of n independent items of the given costs to `parts`
 * devices: assign[i] = device of item i. No reference counterpart (the reference transcribes the
 * pieces of src/split.rs one after another, src/lib.rs:844-900). */
wavo_status wavo_partition_lpt(const uint64_t *cost, uint32_t n, uint32_t parts, uint32_t *assign);

#ifdef __cplusplus
}
#endif

#endif /* WAVO_CUDA_H */
