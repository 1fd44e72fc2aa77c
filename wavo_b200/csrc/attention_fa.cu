// Encoder self-attention without position terms (Whisper, GigaAM after RoPE): the reference's
// `Pass::attention` with qk [q | k | v] or [q | k] + v (src/gpu/mod.rs:1556-1605; attention.wgsl
// `flash`, flash_f16.wgsl), as a tcgen05 flash-attention kernel over segments of any length.
//
// A CTA takes two 128-query tiles of one head of one segment, so that the tensor core works on one
// tile while the other tile's softmax runs:
//   warp 0      TMA: both Q tiles once, then K and V blocks through three-slot rings;
//   warps 1, 2  one thread each issues tile 0's / tile 1's UMMAs: S_t = Q_t·K^T into TMEM, then
//               O_t += P_t·V with P_t read from TMEM (the A operand of a TS UMMA);
//   warps 3-18  softmax, eight warps a tile: two warps share a 32-row quarter of the tile (the TMEM
//               lanes a warp may read), 16 rows each, and two threads of a warp share a row, one
//               half of its key columns each (the 16x32bx2 TMEM access shape). A thread loads its
//               scores from TMEM into registers with one wait, hands the S columns back at once
//               (the next S_t UMMA overlaps this block's exponentials), takes the row maximum
//               with one shuffle, and writes its probabilities back to TMEM as f16 pairs.
// The row maximum lags: the TMEM accumulator is rescaled only when a row maximum grows by more
// than 2^8. Scale/shift and row sums use the paired f32 instructions of sm_100 (fma/add .f32x2).
// At the end the two threads of a row add their sums, normalise and store their halves of O.
//
// Heads of 64: a 128 x 128 block of one tile is 16 384 exponentials against 4 S and 8 P·V UMMAs
// (~640 tensor cycles). The MUFU's 16 exponentials per cycle per SM (measured) make the
// exponentials, not the tensor core, the bound: ~2 050 of the ~2 600 cycles a block pair of the
// two tiles takes (measured), so every exponential goes to the MUFU (an FMA-pipe polynomial for a
// share of them costs more issue slots than the MUFU time it saves; measured). Heads of 128 put
// 6 of 16 on the FMA pipe.
#include "kernels.cuh"
#include "ptx.cuh"
#include "softmax.cuh"

namespace wv {
namespace {

constexpr int BM = 128;
constexpr int NT = 2;                  // query tiles per CTA
constexpr int CTRL_WARPS = 1 + NT;     // TMA producer, one UMMA issuer per tile
constexpr int SOFT_WARPS = 8;          // softmax warps per tile
constexpr int THREADS = 32 * (CTRL_WARPS + NT * SOFT_WARPS);
constexpr int ROPE_WARPS = 4;           // with rotary positions: the warps that rotate Q and K
template <bool ROPE>
constexpr int fa_threads() { return THREADS + (ROPE ? 32 * ROPE_WARPS : 0); }
constexpr int KVS = 3;                 // K and V ring slots

template <int HD, int BN>
struct Fa {
  static constexpr int NBOX = HD / 64;
  static constexpr int ATOM_Q = BM * 128;
  static constexpr int ATOM_KV = BN * 128;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int CW = BN / 2;   // score columns per softmax thread (half a row)
  static constexpr int OW = HD / 2;   // accumulator columns per softmax thread
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NT * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KVS * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + KVS * KV_BYTES;
  // Rotary positions at heads of 64: each K block's table rows (rot <= 64 f32 a key) staged
  // beside it in shared memory, one slot per K slot.
  static constexpr int T_SLOT = BN * 64 * 4;
  static constexpr int OFF_T = OFF_V + KVS * KV_BYTES;
  template <bool ROPE>
  __host__ __device__ static constexpr int off_bar() {
    return ROPE && HD == 64 ? OFF_T + KVS * T_SLOT : OFF_BAR;
  }
  // TMEM columns of tile t, from t·256: the scores S (BN f32 columns), the probabilities P (BN
  // f16, two per column), the accumulator O.
  static constexpr int T_TILE = 256;
  static constexpr int T_S = 0;
  static constexpr int T_P = BN;
  static constexpr int T_O = (BN + BN / 2 + 31) / 32 * 32;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t IDESC_S = idesc_f16(BM, BN, 0);
  static constexpr uint32_t IDESC_PV = idesc_f16(BM, HD, 1);
  static_assert(T_O + HD <= T_TILE && NT * T_TILE <= TMEM_COLS, "TMEM");
  static_assert(CW == 32 || CW == 64, "score columns per thread");
  static_assert(OW % 32 == 0, "accumulator columns per thread");
  static_assert(NT * SOFT_WARPS * 16 * HD * 2 <= 2 * KVS * KV_BYTES, "output staging");
};

struct __align__(8) FaBarriers {
  uint64_t q_full;
  uint64_t q_ready[NT], k_ready[KVS];  // rotary positions: the tile / block is rotated
  uint64_t k_full[KVS], k_empty[KVS];
  uint64_t v_full[KVS], v_empty[KVS];
  uint64_t s_full[NT], s_free[NT];
  uint64_t p_full[NT], pv_done[NT];
  uint64_t o_full;
  uint64_t drain[NT];
  uint32_t tmem_base;
  uint32_t abort;
};

// Rotates one f16 row of a 128-byte-swizzled tile in shared memory ([64-column block][rows][128
// bytes], `atom` bytes a block) by the table row `cs` (rot / 2 cosines, then as many sines): NEOX
// pairs (i, i + rot / 2) or adjacent pairs (2i, 2i + 1), eight columns (one 16-byte chunk) at a
// time; rot / 2 (NEOX) or rot a multiple of 8. The arithmetic of the separate rotary pass:
// a·cos − b·sin, a·sin + b·cos in f32, rounded to f16.
__device__ __forceinline__ uint4 *tile_chunk(uint8_t *tile, int atom, int r, int c) {
  const int cc = c & 63;
  return reinterpret_cast<uint4 *>(tile + (c >> 6) * atom + r * 128 + (((cc >> 3) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void rot_pair(__half &x0, __half &x1, float c, float s) {
  const float a = __half2float(x0), b = __half2float(x1);
  x0 = __float2half_rn(a * c - b * s);
  x1 = __float2half_rn(a * s + b * c);
}

// One rotation unit: 8 NEOX pairs (chunk i of the first half with chunk i + half) or 4 adjacent
// pairs (chunk c), at column `col` of row r. Loads first, then the arithmetic, so that a thread's
// table reads of several units are in flight together.
struct RopeUnit {
  uint4 lo, hi;
  float4 c0, c1, s0, s1;
};

__device__ __forceinline__ void rope_load(RopeUnit &u, uint8_t *tile, int atom, int r, int col,
                                          const float *cs, int half, bool neox) {
  if (neox) {
    u.lo = *tile_chunk(tile, atom, r, col);
    u.hi = *tile_chunk(tile, atom, r, col + half);
    u.c0 = *reinterpret_cast<const float4 *>(cs + col);
    u.c1 = *reinterpret_cast<const float4 *>(cs + col + 4);
    u.s0 = *reinterpret_cast<const float4 *>(cs + half + col);
    u.s1 = *reinterpret_cast<const float4 *>(cs + half + col + 4);
  } else {
    u.lo = *tile_chunk(tile, atom, r, col);
    u.c0 = *reinterpret_cast<const float4 *>(cs + col / 2);
    u.s0 = *reinterpret_cast<const float4 *>(cs + half + col / 2);
  }
}

__device__ __forceinline__ void rope_store(RopeUnit &u, uint8_t *tile, int atom, int r, int col,
                                           int half, bool neox) {
  if (neox) {
    const float cc[8] = {u.c0.x, u.c0.y, u.c0.z, u.c0.w, u.c1.x, u.c1.y, u.c1.z, u.c1.w};
    const float ss[8] = {u.s0.x, u.s0.y, u.s0.z, u.s0.w, u.s1.x, u.s1.y, u.s1.z, u.s1.w};
    __half *l = reinterpret_cast<__half *>(&u.lo), *h = reinterpret_cast<__half *>(&u.hi);
#pragma unroll
    for (int k = 0; k < 8; ++k) rot_pair(l[k], h[k], cc[k], ss[k]);
    *tile_chunk(tile, atom, r, col) = u.lo;
    *tile_chunk(tile, atom, r, col + half) = u.hi;
  } else {
    const float cc[4] = {u.c0.x, u.c0.y, u.c0.z, u.c0.w}, ss[4] = {u.s0.x, u.s0.y, u.s0.z, u.s0.w};
    __half *e = reinterpret_cast<__half *>(&u.lo);
#pragma unroll
    for (int k = 0; k < 4; ++k) rot_pair(e[2 * k], e[2 * k + 1], cc[k], ss[k]);
    *tile_chunk(tile, atom, r, col) = u.lo;
  }
}

// Rotates units part, part + parts, .. of row r (table row cs), two units at a time.
__device__ void rope_tile_row(uint8_t *tile, int atom, int r, const float *cs, int rot,
                              bool neox, int part, int parts) {
  const int half = rot / 2;
  const int units = neox ? half / 8 : rot / 8;
#pragma unroll 1
  for (int k = part; k < units; k += 2 * parts) {
    const bool two = k + parts < units;
    RopeUnit u0, u1;
    rope_load(u0, tile, atom, r, 8 * k, cs, half, neox);
    if (two) rope_load(u1, tile, atom, r, 8 * (k + parts), cs, half, neox);
    rope_store(u0, tile, atom, r, 8 * k, half, neox);
    if (two) rope_store(u1, tile, atom, r, 8 * (k + parts), half, neox);
  }
}

// KS: K-steps of 16 columns in a score UMMA group (the head's width in 16s; all HD / 16 when the
// host zero-padded the heads). ROPE: rotary positions on q and k (a.rope_table), applied to each Q
// tile and K block in shared memory by four more warps before the UMMAs read them.
template <int HD, int BN, int KS, bool ROPE>
__global__ void __launch_bounds__(fa_threads<ROPE>(), 1)
    fa_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_kv,
              const __grid_constant__ CUtensorMap map_o, const AttnArgs a) {
  using C = Fa<HD, BN>;
  constexpr int CW = C::CW, OW = C::OW;
  const int seg = blockIdx.z, h = blockIdx.y;
  const int T = a.seg_len ? a.seg_len[seg] : a.single_t;
  const int row0 = a.seg_len ? a.seg_start[seg] : 0;
  const int m0 = blockIdx.x * (NT * BM);
  if (m0 >= T) return;  // uniform: the whole CTA leaves before any setup
  const int nt = (m0 + BM < T) ? NT : 1;  // tiles with queries in the segment
  const int nb = (T + BN - 1) / BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  FaBarriers *bar = reinterpret_cast<FaBarriers *>(smem + C::template off_bar<ROPE>());
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int t = 0; t < NT; ++t) mbar_init(&bar->q_ready[t], SOFT_WARPS);
    for (int i = 0; i < KVS; ++i) {
      mbar_init(&bar->k_ready[i], ROPE_WARPS);
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], nt);  // one commit from each live tile's issuer
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], nt);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&bar->s_full[t], 1);
      mbar_init(&bar->s_free[t], SOFT_WARPS);
      mbar_init(&bar->p_full[t], SOFT_WARPS);
      mbar_init(&bar->pv_done[t], 1);
      mbar_init(&bar->drain[t], 1);
    }
    mbar_init(&bar->o_full, nt);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_kv);
    if (a.o_tma) prefetch_tmap(&map_o);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, a.err};
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  const int hoff = h * a.head_stride;

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      uint32_t k_last[KVS] = {}, v_last[KVS] = {};  // bit 1: armed; bit 0: parity
      mbar_arrive_expect_tx(&bar->q_full, nt * C::Q_BYTES);
      for (int t = 0; t < nt; ++t)
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_Q + t * C::Q_BYTES + b * C::ATOM_Q, &map_q, &bar->q_full,
                      a.q_off + hoff + 64 * b, row0 + m0 + t * BM);
      for (int j = 0; j < nb; ++j) {
        const int s = j % KVS;
        const uint32_t par = ((j / KVS) & 1) ^ 1u;
        if (!mbar_wait(&bar->k_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
        // Rotary positions at heads of 64: the table rows of the block's keys in the segment
        // (contiguous, rot f32 each) come with K on the same barrier.
        const uint32_t tbytes =
            ROPE && HD == 64 ? uint32_t(min(BN, T - j * BN) * a.rope_rot * 4) : 0u;
        mbar_arrive_expect_tx(&bar->k_full[s], C::KV_BYTES + tbytes);
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_K + s * C::KV_BYTES + b * C::ATOM_KV, &map_kv, &bar->k_full[s],
                      a.k_off + hoff + 64 * b, row0 + j * BN);
        if (tbytes)
          bulk_load(smem + C::OFF_T + s * C::T_SLOT,
                    a.rope_table + (long long)(a.rope_pos + j * BN) * a.rope_rot, tbytes,
                    &bar->k_full[s]);
        k_last[s] = 2u | ((j / KVS) & 1u);
        if (!mbar_wait(&bar->v_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar->v_full[s], C::KV_BYTES);
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_V + s * C::KV_BYTES + b * C::ATOM_KV, &map_kv, &bar->v_full[s],
                      a.v_off + hoff + 64 * b, row0 + j * BN);
        v_last[s] = 2u | ((j / KVS) & 1u);
      }
      if (!ok) {
        const long long t0 = clock64();
        auto drain = [&](uint64_t *b, uint32_t last) {
          if (!(last & 2u)) return;
          while (!mbar_try_wait(b, last & 1u) && clock64() - t0 < kWaitCycles) {
          }
        };
        drain(&bar->q_full, 2u);
        for (int s = 0; s < KVS; ++s) {
          drain(&bar->k_full[s], k_last[s]);
          drain(&bar->v_full[s], v_last[s]);
        }
      }
    }
  } else if (warp < CTRL_WARPS) {
    // ---- UMMA issuer of tile t -------------------------------------------------------------
    // Per block j: S_t(j) = Q_t·K(j)^T as soon as the tile's softmax holds S_t(j-1) in registers,
    // then O_t += P_t(j-1)·V(j-1) once P_t(j-1) is in TMEM. One issuing thread per tile, so that
    // one thread's barrier waits and commits overlap the other tile's UMMAs.
    const int t = int(warp) - 1;
    if (lane == 0 && t < nt) {
      bool ok = mbar_wait(ROPE ? &bar->q_ready[t] : &bar->q_full, 0, ab, kErrTimeoutMma);
      bool issued = false;
      // Descriptors are linear in the start address (bits 0-13 hold address / 16), so every
      // operand's descriptor is a base plus an offset / 16. The score loop is unrolled over a
      // compile-time count of K-steps and issues every UMMA unconditionally: the same loop with a
      // guard on each UMMA (k-step < the head's steps) produced wrong scores; the unguarded and
      // the rolled forms are exact.
      const uint64_t dq = sdesc_sw128(smem_u32(smem + C::OFF_Q + t * C::Q_BYTES), 16, 1024);
      const uint64_t dk = sdesc_sw128(smem_u32(smem + C::OFF_K), 16, 1024);
      const uint64_t dv = sdesc_sw128(smem_u32(smem + C::OFF_V), C::ATOM_KV, 1024);
      const uint32_t tt = tmem + t * C::T_TILE;
      tc_fence_after();
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          const int ks = j % KVS;
          if (!mbar_wait(ROPE ? &bar->k_ready[ks] : &bar->k_full[ks], (j / KVS) & 1, ab,
                         kErrTimeoutMma)) {
            ok = false;
            break;
          }
          if (j >= 1 && !mbar_wait(&bar->s_free[t], (j - 1) & 1, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bk0 = dk + uint64_t((ks * C::KV_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < KS; ++kk) {
            const uint32_t o_q = ((kk >> 2) * C::ATOM_Q + (kk & 3) * 32) >> 4;
            const uint32_t o_k = ((kk >> 2) * C::ATOM_KV + (kk & 3) * 32) >> 4;
            umma_f16(tt + C::T_S, dq + o_q, bk0 + o_k, C::IDESC_S, kk > 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&bar->s_full[t]);
          umma_commit(&bar->k_empty[ks]);
        }
        if (j >= 1) {
          const int i = j - 1, vs = i % KVS;
          if (!mbar_wait(&bar->v_full[vs], (i / KVS) & 1, ab, kErrTimeoutMma) ||
              !mbar_wait(&bar->p_full[t], i & 1, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bv0 = dv + uint64_t((vs * C::KV_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            // A = P from TMEM: keys 16kk.. are columns 8kk.. of the P region; B = V rows 16kk..
            umma_f16_ts(tt + C::T_O, tt + C::T_P + kk * 8, bv0 + uint64_t((kk * 16 * 128) >> 4),
                        C::IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bar->pv_done[t]);
          umma_commit(&bar->v_empty[vs]);
        }
      }
      if (ok) {
        umma_commit(&bar->o_full);
      } else if (issued) {
        umma_commit(&bar->drain[t]);
        const long long t0 = clock64();
        while (!mbar_try_wait(&bar->drain[t], 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (ROPE && warp >= CTRL_WARPS + NT * SOFT_WARPS) {
    // ---- rotary positions: thread t rotates rows t, t + 128, .. of each K block as it lands (key
    // j of the segment at table row rope_pos + j); rows past the segment are left as they are
    // (their keys are masked). The softmax warps rotate their tile's Q rows at the start.
    const int t = int(threadIdx.x) - 32 * (CTRL_WARPS + NT * SOFT_WARPS);
    const int rot = a.rope_rot;
    const bool neox = a.rope_neox != 0;
    for (int j = 0; j < nb; ++j) {
      const int ks = j % KVS;
      if (!mbar_wait_warp(&bar->k_full[ks], (j / KVS) & 1, ab, kErrTimeoutConsumer)) break;
      for (int r = t; r < BN; r += 32 * ROPE_WARPS) {
        const int kj = j * BN + r;
        if (kj < T)
          rope_tile_row(smem + C::OFF_K + ks * C::KV_BYTES, C::ATOM_KV, r,
                        HD == 64 ? reinterpret_cast<const float *>(smem + C::OFF_T + ks * C::T_SLOT) +
                                       r * rot
                                 : a.rope_table + (long long)(a.rope_pos + kj) * rot,
                        rot, neox, 0, 1);
      }
      fence_proxy_async_smem();  // the rotated rows are visible to the UMMAs (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->k_ready[ks]);
    }
  } else {
    // ---- softmax: 8 warps a tile. The two warps of a quarter (the TMEM lanes 32·(w % 4) a warp
    // may access) take 16 rows each; within a warp, threads t and t + 16 share row t % 16 and hold
    // its two halves of the key columns (the 16x32bx2 TMEM access shape), so a row maximum or sum
    // needs one shuffle.
    const int w = int(warp) - CTRL_WARPS;
    const int t = w >> 3, sub = (w >> 2) & 1;
    const uint32_t quarter = warp & 3u;
    const int ch = int(lane >> 4);  // column half of this thread
    const uint32_t tl = tmem + ((quarter * 32u + sub * 16u) << 16) + t * C::T_TILE;
    const uint32_t ts = tl + C::T_S, tp = tl + C::T_P, to = tl + C::T_O;
    const float c = a.scale_log2;
    float m_use = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    bool ok = t < nt;
    if (ROPE && ok) {
      // The tile's 128 Q rows, two threads a row (alternate rotation units), before its issuer's
      // first UMMA (query i of the segment at table row rope_pos + i).
      ok = mbar_wait_warp(&bar->q_full, 0, ab, kErrTimeoutConsumer);
      if (ok) {
        const int tw = (w & 7) * 32 + int(lane);  // 0..255 within the tile's softmax warps
        const int r = tw >> 1, qi = m0 + t * BM + r;
        if (qi < T)
          rope_tile_row(smem + C::OFF_Q + t * C::Q_BYTES, C::ATOM_Q, r,
                        a.rope_table + (long long)(a.rope_pos + qi) * a.rope_rot, a.rope_rot,
                        a.rope_neox != 0, tw & 1, 2);
        fence_proxy_async_smem();  // the rotated rows are visible to the UMMAs (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->q_ready[t]);
      }
    }
    for (int j = 0; j < nb && ok; ++j) {
      if (!mbar_wait_warp(&bar->s_full[t], j & 1, ab, kErrTimeoutConsumer)) { ok = false; break; }
      tc_fence_after();
      float s[CW];
      {
        uint32_t r[32];
        tmem_ld_16x2_x32<CW>(ts, r);
        if constexpr (CW == 64) {
          uint32_t r2[32];
          tmem_ld_16x2_x32<CW>(ts + 32, r2);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) s[32 + x] = __uint_as_float(r2[x]);
        } else {
          tmem_wait_ld();
        }
#pragma unroll
        for (int x = 0; x < 32; ++x) s[x] = __uint_as_float(r[x]);
      }
      // The scores are in registers: the issuer may overwrite S with the next block's.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->s_free[t]);
      // Keys past the segment (last block only) are masked to -inf.
      const int kvalid = T - j * BN - ch * CW;
      if (kvalid < CW) {
#pragma unroll
        for (int x = 0; x < CW; ++x)
          if (x >= kvalid) s[x] = -INFINITY;
      }
      float mx;
      {
        // Four independent chains of 3-input maxima, then the other half of the row.
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int x = 0; x < CW; x += 8) {
          float &m = m4[(x / 8) & 3];
          m = max3(m, s[x + 0], s[x + 1]);
          m = max3(m, s[x + 2], s[x + 3]);
          m = max3(m, s[x + 4], s[x + 5]);
          m = max3(m, s[x + 6], s[x + 7]);
        }
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      }
      const float m_blk = mx * c;
      const bool need = m_blk > m_use + 8.0f;
      const bool rescale = __any_sync(0xffffffffu, need) && j > 0;
      const float alpha = need ? ex2(m_use - m_blk) : 1.0f;
      if (rescale) {
        l0 *= alpha;
        l1 *= alpha;
      }
      if (need) m_use = m_blk;
      const float nm = -m_use;
      // Probabilities: 16 at a time, 6 of them on the FMA pipe.
      uint32_t pk[CW / 2];
#pragma unroll
      for (int g = 0; g < CW; g += 16) {
        float *p = s + g;  // in place: scores become exponents, then probabilities
#pragma unroll
        for (int x = 0; x < 16; x += 2) fma2(p[x], p[x + 1], p[x], p[x + 1], c, c, nm, nm);
        exp2_16<(HD == 64 ? 0 : 6)>(p);
#pragma unroll
        for (int x = 0; x < 16; x += 4) {
          float a0, a1;
          add2(a0, a1, p[x], p[x + 1], p[x + 2], p[x + 3]);
          add2(l0, l1, l0, l1, a0, a1);
        }
#pragma unroll
        for (int x = 0; x < 8; ++x) pk[g / 2 + x] = pack_half2(p[2 * x], p[2 * x + 1]);
      }
      // P_t is free and O_t stable once P·V of block j - 1 landed.
      if (j >= 1 && !mbar_wait_warp(&bar->pv_done[t], (j - 1) & 1, ab, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if constexpr (CW == 64) {
        tmem_st_16x2_x32<CW / 2>(tp, pk);
      } else {
        tmem_st_16x2_x16<CW / 2>(tp, pk);
      }
      if (rescale) {
#pragma unroll 1
        for (int q = 0; q < OW / 16; ++q) {
          uint32_t r[16];
          tmem_ld_16x2_x16<OW>(to + q * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 16; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * alpha);
          tmem_st_16x2_x16<OW>(to + q * 16, r);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full[t]);
    }
    if (ok && mbar_wait_warp(&bar->o_full, 0, ab, kErrTimeoutConsumer)) {
      // The row sum over both halves, then this thread's half of the row of O.
      float l = l0 + l1;
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      tc_fence_after();
      const float inv = 1.0f / l;
      const int rbase = m0 + t * BM + int(quarter * 32u + sub * 16u);  // this warp's 16 rows
      const int qrow = rbase + int(lane & 15u);
      const bool store = qrow < T;
      // A warp whose 16 rows all lie in the segment stages them in shared memory (the K ring,
      // free once O is final: every load landed and every UMMA completed) and stores them with
      // one TMA box; the segment's last partial group is stored row by row.
      const bool via_tma = a.o_tma && rbase + 16 <= T;
      uint8_t *stage = smem + C::OFF_K + w * (16 * HD * 2) + (lane & 15u) * (a.hd * 2);
      const long long orow = (long long)(row0 + qrow) * a.ldo + (long long)h * a.hd;
#pragma unroll
      for (int q = 0; q < OW / 32; ++q) {
        uint32_t r[32];
        tmem_ld_16x2_x32<OW>(to + q * 32, r);
        tmem_wait_ld();
        const int c0 = ch * OW + q * 32;
        if (via_tma) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            if (c0 + x < a.hd) {  // the head size is a multiple of 8 on this path
              const uint4 v = make_uint4(
                  pack_half2(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv),
                  pack_half2(__uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv),
                  pack_half2(__uint_as_float(r[x + 4]) * inv, __uint_as_float(r[x + 5]) * inv),
                  pack_half2(__uint_as_float(r[x + 6]) * inv, __uint_as_float(r[x + 7]) * inv));
              *reinterpret_cast<uint4 *>(stage + (c0 + x) * 2) = v;
            }
          }
        } else if (store && c0 < a.hd) {
          if (a.o_f16) {
            __half *o = reinterpret_cast<__half *>(a.o) + orow;
            if (c0 + 32 <= a.hd && ((reinterpret_cast<uintptr_t>(o + c0) & 15u) == 0)) {
#pragma unroll
              for (int x = 0; x < 32; x += 8) {
                const uint4 v = make_uint4(
                    pack_half2(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv),
                    pack_half2(__uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv),
                    pack_half2(__uint_as_float(r[x + 4]) * inv, __uint_as_float(r[x + 5]) * inv),
                    pack_half2(__uint_as_float(r[x + 6]) * inv, __uint_as_float(r[x + 7]) * inv));
                *reinterpret_cast<uint4 *>(o + c0 + x) = v;
              }
            } else {
#pragma unroll
              for (int x = 0; x < 32; ++x)
                if (c0 + x < a.hd) o[c0 + x] = __float2half_rn(__uint_as_float(r[x]) * inv);
            }
          } else {
            float *o = reinterpret_cast<float *>(a.o) + orow;
#pragma unroll
            for (int x = 0; x < 32; ++x)
              if (c0 + x < a.hd) o[c0 + x] = __uint_as_float(r[x]) * inv;
          }
        }
      }
      if (via_tma) {
        fence_proxy_async_smem();  // the staged rows are visible to the TMA (async proxy)
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_o, smem + C::OFF_K + w * (16 * HD * 2), h * a.hd, row0 + rbase);
          bulk_commit();
          // Shared memory may go once the TMA has read it; the writes complete with the grid.
          bulk_wait_read<0>();
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int HD, int BN, int KS, bool ROPE>
cudaError_t launch_fa(const CUtensorMap &q, const CUtensorMap &kv, const CUtensorMap &o,
                      const AttnArgs &a, int max_len, int nseg, cudaStream_t s) {
  using C = Fa<HD, BN>;
  const size_t smem = 1024 + C::template off_bar<ROPE>() + sizeof(FaBarriers);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fa_kernel<HD, BN, KS, ROPE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid((max_len + NT * BM - 1) / (NT * BM), a.heads, nseg);
  return launch_pdl(fa_kernel<HD, BN, KS, ROPE>, grid, dim3(fa_threads<ROPE>()), smem, s, q, kv, o,
                    a);
}

}  // namespace

int fa_block_keys(int hd_pad) { return hd_pad == 64 ? 128 : 64; }

cudaError_t launch_fa_attention(const CUtensorMap &map_q, const CUtensorMap &map_kv,
                                const CUtensorMap &map_o, const AttnArgs &a, int hd_pad,
                                int max_len, int nseg, cudaStream_t s) {
  if (max_len <= 0 || nseg <= 0) return cudaSuccess;
  // Heads read in place (a head stride below 64): the head's own K-steps; zero-padded heads: all.
  const int ks = a.head_stride < 64 ? (a.hd + 15) / 16 : 4;
  if (a.rope_table) {
    if (hd_pad == 128) return launch_fa<128, 64, 8, true>(map_q, map_kv, map_o, a, max_len, nseg, s);
    switch (ks) {
      case 1: return launch_fa<64, 128, 1, true>(map_q, map_kv, map_o, a, max_len, nseg, s);
      case 2: return launch_fa<64, 128, 2, true>(map_q, map_kv, map_o, a, max_len, nseg, s);
      case 3: return launch_fa<64, 128, 3, true>(map_q, map_kv, map_o, a, max_len, nseg, s);
      default: return launch_fa<64, 128, 4, true>(map_q, map_kv, map_o, a, max_len, nseg, s);
    }
  }
  if (hd_pad == 128) return launch_fa<128, 64, 8, false>(map_q, map_kv, map_o, a, max_len, nseg, s);
  switch (ks) {
    case 1: return launch_fa<64, 128, 1, false>(map_q, map_kv, map_o, a, max_len, nseg, s);
    case 2: return launch_fa<64, 128, 2, false>(map_q, map_kv, map_o, a, max_len, nseg, s);
    case 3: return launch_fa<64, 128, 3, false>(map_q, map_kv, map_o, a, max_len, nseg, s);
    default: return launch_fa<64, 128, 4, false>(map_q, map_kv, map_o, a, max_len, nseg, s);
  }
}

}  // namespace wv
