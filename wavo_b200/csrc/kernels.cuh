// Launch interfaces of the library's kernels (host side). The C ABI in wavo_cuda.cu validates the
// arguments and builds the tensor maps; these functions only configure and launch.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace wv {

// Launches `kernel` with programmatic stream serialization: it may begin (and set itself up) while
// the previous kernel of the stream is still running; the kernel itself waits for that grid
// (griddepcontrol.wait) before it touches any data. Only kernels that do so are launched here.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Epilogue modes, the reference's `Epilogue` (src/gpu/mod.rs:431-456) in its kernel order.
enum Epi : int { kBias = 0, kSilu, kRelu, kResidual, kGelu, kGeluResidual, kTanh };

// ---- projection GEMM (gemm.cu) ----------------------------------------------------------

struct GemmArgs {
  int m;              // rows of a and c
  int cols;           // main output columns
  int dual;           // leading outputs written a second time at cols.. with bias[cols + j]
  int k;              // inner dimension
  const float *bias;  // at least max(cols, cols + dual) floats
  void *c;
  long long ldc;      // elements
  int c_f16;          // 1: c is f16, 0: f32
  int epilogue;
  float alpha;
  int *err;           // device error word
  int c_tma;          // pair GEMM: store c through the tensor map tma_c (no dual outputs; f32 when
                      // the epilogue adds into c: a TMA reduce-add)
};

constexpr int kGemmBM = 128, kGemmBK = 64;
constexpr int kGemmThreads = 192;
// kc: 64-column K chunks per pipeline stage. kc = 1 takes 2D tensor maps with boxes {64, rows};
// kc = 2 takes 3D maps {64, rows, k / 64} (k a multiple of 64, chunk stride 128 bytes) with boxes
// {64, rows, 2}. Tile width (128, 160 or 256) for an m x cols output on num_sms SMs; the W tensor
// map's box height.
int gemm_pick_bn(int m, int cols, int num_sms);
cudaError_t launch_gemm(const CUtensorMap &a, const CUtensorMap &w, const GemmArgs &g, int bn,
                        int kc, int num_sms, cudaStream_t s);
// The Q8_0 GEMM (W dequantised in the prologue): q is an int8 tensor map over W's block values
// [rows][k] (boxes {64, bn}, no swizzle), sc an f16 map over the scales transposed, [k / 32][rows]
// (boxes {bn, 2}). Tile widths as gemm_pick_bn.
cudaError_t launch_gemm_q8(const CUtensorMap &a, const CUtensorMap &q, const CUtensorMap &sc,
                           const GemmArgs &g, int bn, int num_sms, cudaStream_t s);
// The pair GEMM (a cluster of two CTAs shares each UMMA of M=256): tile width BN (128, 160, 192
// or 256) for an m x cols output; a's box height is 128 and W's BN / 2.
int gemm2_pick_bn(int m, int cols, int num_sms);
// tma_c (with g.c_tma): c as a 2D tensor {cols, m}, boxes {32, 32}, 128-byte swizzle for f32 and
// 64-byte swizzle for f16.
cudaError_t launch_gemm2(const CUtensorMap &a, const CUtensorMap &w_half, const CUtensorMap &tma_c,
                         const GemmArgs &g, int bn, int kc, int num_sms, cudaStream_t s);

// f32 rows -> f16 rows (round to nearest even), into a padded row stride; columns past `cols`
// up to `ld_out` are zeroed.
cudaError_t launch_cast_rows(const float *in, long long ld_in, __half *out, long long ld_out,
                             int rows, int cols, cudaStream_t s);

// ---- encoder attention (attention.cu) ----------------------------------------------------

struct AttnArgs {
  // Segments: segment z covers rows seg_start[z] .. seg_start[z] + seg_len[z] of every operand.
  // With seg_len == nullptr there is one segment of single_t rows from row 0.
  const int *seg_start;
  const int *seg_len;
  int single_t;
  int heads;
  int hd;           // real head size
  int head_stride;  // elements between heads inside a section of the f16 operand rows
  int q_off, k_off, v_off, qv_off;  // section offsets (elements) inside the operand rows
  int pos_off;      // head offset base inside the position rows
  int pos_t;        // the position table's t: row r is relative position pos_t + 15 - r
  float scale_log2; // log2(e) / sqrt(hd)
  void *o;          // output rows
  long long ldo;
  int o_f16;
  int o_tma;        // 1: f16 output rows also reachable through map_o (boxes {hd, 16}, no swizzle)
  int *err;
  // Rotary positions on q and k inside the plain kernel (rope_table NULL: none): row i of a
  // segment takes table row rope_pos + i (rope_rot / 2 cosines, then as many sines); NEOX pairs
  // (i, i + rot / 2) or adjacent pairs.
  const float *rope_table;
  int rope_rot, rope_neox, rope_pos;
};

// ---- encoder block around the attention (encoder.cu) ----
enum { kLnNorm = 0, kLnNormSilu = 1, kLnAffineSilu = 2 };
// Row-wise LayerNorm of f32 x [rows][cols] into y (f16 or f32); mode kLnNormSilu adds SiLU,
// kLnAffineSilu is w·x + b then SiLU; with a table, yr = y with NEOX rotary pairs inside heads of hd
// (table row positions[r], or r).
cudaError_t launch_layer_norm(const float *x, const float *w, const float *b, void *y, int y_f16,
                              int rows, int cols, int mode, const float *table,
                              const int *positions, void *yr, int hd, cudaStream_t s);
int layer_norm_max_cols();
// GLU of h [rows][2ch] and the depthwise conv over each segment's frames into z [rows][ch] f32
// (taps [ch][kernel], odd kernel, centred); with n_w (an affine norm) y = SiLU(n_w·z + n_b) into z
// instead, f16 when y_f16.
cudaError_t launch_dwconv(const float *h, const float *taps, const float *bias, void *z, int ch,
                          int kernel, const int *seg_start, const int *seg_len, int nseg,
                          int max_len, const float *n_w, const float *n_b, int y_f16,
                          cudaStream_t s);
int dwconv_max_kernel();

// ---- the decoder step's ends (decoder.cu) ----
// x[b] = W[tokens[b]] + positions[pos] + bias for b < rows (wtype 0: f32 W, 1: f16, 8: int8 with
// f32 scales d8 a block of 32); positions may be NULL.
cudaError_t launch_embed(const void *w, int wtype, const float *d8, const float *bias,
                         const float *positions, const int *tokens, int rows, int k, int pos,
                         float *x, long long ldx, cudaStream_t s);
// Greedy pick with Whisper's suppression and timestamp rules, one CTA a row (see decoder.cu).
cudaError_t launch_pick(float *logits, long long ld, int rows, int vocab, int *history,
                        int *hist_len, int max_hist, const int *suppress, int n_suppress,
                        const int *begin_suppress, int n_begin, int eot, int no_ts, int begin,
                        int max_initial, int *tokens, float *logprobs, cudaStream_t s);

constexpr int kAttnBlockQ = 128;  // queries per tile (the TMA box height of map_q)
int attn_block_keys(bool rel, int hd_pad);  // keys per block (the TMA box height of map_kv)
int attn_pos_window_rows();      // position rows per block (the TMA box height of map_pos)
// The plain-layout kernel (attention_fa.cu): two query tiles per CTA.
int fa_block_keys(int hd_pad);
cudaError_t launch_fa_attention(const CUtensorMap &map_q, const CUtensorMap &map_kv,
                                const CUtensorMap &map_o, const AttnArgs &a, int hd_pad,
                                int max_len, int nseg, cudaStream_t s);
// hd_pad: 64 or 128 (the padded head size of the operand tiles). Plain attention takes 2D f16
// tensor maps with 64-column (128-byte) boxes; relative attention (heads of 128) 3D maps
// {64, rows, columns / 64} with boxes {64, rows, 2}; all with 128-byte swizzle. map_o (read with
// a.o_tma): the f16 output as a 2D tensor {heads * hd, rows}, boxes {hd, 16}, no swizzle.
cudaError_t launch_attention(const CUtensorMap &map_q, const CUtensorMap &map_kv,
                             const CUtensorMap &map_pos, const CUtensorMap &map_o,
                             const AttnArgs &a, int hd_pad, bool rel, int max_len, int nseg,
                             cudaStream_t s);

// Repacks attention operands into f16 rows with heads padded to `hd_pad` (zeros past hd):
// out[row][sec * heads * hd_pad + h * hd_pad + c] = in[row][in_off[sec] + h * hd + c], for
// `sections` sections. `in_f16` selects the input type.
cudaError_t launch_pack_heads(const void *in, int in_f16, long long ld_in, const int *in_off,
                              int sections, __half *out, long long ld_out, int rows, int heads,
                              int hd, int hd_pad, cudaStream_t s);

// ---- decoder (decode.cu) -----------------------------------------------------------------

cudaError_t launch_pack_cache(const float *x, long long src, long long stride, uint32_t *cache,
                              int rows, int d, int cols, int col, long long x_batch,
                              long long cache_batch, int batch, cudaStream_t s);
cudaError_t launch_attend(const float *q, long long q_stride, const uint32_t *kv,
                          long long kv_stride, float *part, float *o, long long o_stride, int n,
                          int cols, int heads, int hd, int batch, cudaStream_t s);
size_t attend_part_floats(int n, int heads, int hd, int batch);
// positions (device, optional): the table row of each row; without it row r uses pos + r.
cudaError_t launch_rope(const float *table, void *qkv, int x_f16, long long stride, int rows,
                        int pos, const int *positions, int heads, int hd, int rot, int neox,
                        int sections, cudaStream_t s);
// Rows (<= 32) of f32 a through W of type wtype (0 f32 [n][k], 1 f16 [n][k], 8 int8 [n][k] with
// f32 scales [n][k/32]) in f32: the reference's gemv (W not rounded to f16).
// F16 weights, any epilogue, rows <= 32: the tensor-core gemv (split f16 rows of a, f32 accuracy)
// over W's 128-row 2D tensor map and a's map of f32 {64, 32} boxes (make_map_rows32).
cudaError_t launch_gemv_tc(const CUtensorMap &map_a, const CUtensorMap &map_w128,
                           const float *bias, float *c, long long ldc, int rows, int n, int k,
                           int epilogue, float alpha, int sms, int *err, cudaStream_t s);
cudaError_t launch_gemv(const float *a, long long lda, int wtype, const void *w,
                        const float *scales, const float *bias, float *c, long long ldc, int rows,
                        int n, int k, int epilogue, float alpha, cudaStream_t s);

// ---- the log-mel frontend (frontend.cu) ----------------------------------------------------------

// Device tables of the frontend, one image that the log-mel kernel copies into shared memory: the
// FFT's twiddles and first-stage order, the Hann window in that order, and the Slaney filterbank
// as each mel bin's nonzero span of FFT bins.
struct FrontendTables {
  const void *image;
  unsigned *count;  // the log-mel CTAs that have published their sums (0 between launches)
};
size_t frontend_table_bytes();
// Fills `dev` (frontend_table_bytes()) with the tables and points `out` at them (waits for `s`).
cudaError_t frontend_tables_upload(void *dev, cudaStream_t s, FrontendTables *out);
// mel [frames][128] = the log-mel of frames f0 .. f0 + frames of the 16 kHz pcm (n_pcm samples).
cudaError_t launch_log_mel(const float *pcm, long long n_pcm, long long f0, int frames,
                           const FrontendTables &tab, float *mel, cudaStream_t s);
// Each mel bin normalised over frames 0 .. frames - 2, the last frame zeroed (frames >= 3).
// mel [frames][128] = the normalised log-mel features of all frames of the pcm (frames =
// n_pcm / 160 + 1 ≥ 3): each bin less its mean over all frames but the last, times 1 / (the
// unbiased std + 1e-5); the last frame zero. scratch: mel_features_scratch_bytes(sms) bytes, sms =
// the device's SM count.
size_t mel_features_scratch_bytes(int sms);
cudaError_t launch_mel_features(const float *pcm, long long n_pcm, int frames,
                                const FrontendTables &tab, float *mel, void *scratch, int sms,
                                cudaStream_t s);

// Parakeet's subsampling around its GEMMs, each output the next GEMM's f16 operand: conv0 + ReLU
// + conv2 from the mel image into a [t2][32][ch] (rows from half(half(valid)) on zero); a depthwise
// 3x3 stride-2 conv of x [t][f][ch] into y [rows][half(f)][ch]; [t][f][ch] to [t][ch·f].
cudaError_t launch_conv02(const float *mel, int valid, int t2, int ch, const float *w0,
                          const float *b0, const float *w2, const float *b2, __half *a,
                          cudaStream_t s);
cudaError_t launch_dw3s2(const float *x, int t, int f, int ch, int rows, const float *w,
                         const float *b, __half *y, cudaStream_t s);
cudaError_t launch_flatten(const float *y, int t, int f, int ch, __half *h, cudaStream_t s);

// ---- GGUF loads (gguf.cu) ----------------------------------------------------------------------

// Raw Q8_0 blocks of rows x k weights into q8 [n][k] int8, d8 [n][k/32] f32, s16t [k/32][n] f16 and
// w16 [n][k] f16 (q·d rounded); rows past `rows` are left as they are (the caller zeroes them).
cudaError_t launch_build_q8(const uint8_t *raw, int rows, int k, int n, int8_t *q8, float *d8,
                            __half *s16t, __half *w16, cudaStream_t s);
// w16[i] = f16(w32[i]) for i < count (count a multiple of 4).
cudaError_t launch_build_f16(const float *w32, long long count, __half *w16, cudaStream_t s);

// ---- self-checks (selftest.cu) -------------------------------------------------------------

// One warp waits on an mbarrier nothing arms, giving up after `limit` cycles (raises *err).
cudaError_t launch_wait_probe(int *err, long long limit, cudaStream_t s);
// y[i] = 2^x[i] by the softmax's FMA-pipe polynomial (x in [-125, 8]).
cudaError_t launch_exp2_probe(const float *x, float *y, int n, cudaStream_t s);

}  // namespace wv
