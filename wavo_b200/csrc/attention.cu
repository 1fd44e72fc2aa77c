// Encoder multi-head attention with relative positions (Transformer-XL, Parakeet): the reference's
// `Pass::attention` with [q+u | k | v | q+v] rows and a position table (src/gpu/mod.rs:1556-1605;
// attention.wgsl `relative`, src/cpu/ops.rs:223-273), as a tcgen05 flash-attention kernel over
// segments of any length in one launch. score(i, j) = ((q+u)_i·k_j + (q+v)_i·P[pos_t + 15 - (i - j)])
// / sqrt(hd).
//
// Persistent: one CTA per SM walks its share of the work items (128 queries of one head of one
// segment; items dealt round-robin over tile, head, segment), each item's keys in blocks of 64, with
// the ring slots and barrier phases running on across items, so that the next item's loads and
// first scores overlap the current item's last block and epilogue:
//   warp 0      TMA: Q and Q+v (once the previous item's last scores have read them), then K, V
//               and position windows through two-slot rings, each a single 3D box of the head's
//               two 64-column chunks;
//   warp 1      one thread issues BD' = (q+v)·window^T over the 191 position rows a 128 x 64
//               block needs (one N=192 UMMA group) and AC = (q+u)·K^T (N=64);
//   warp 2      one thread issues O += P·V with P read from TMEM (TS UMMAs, N=128);
//   warps 3-10  softmax, eight warps: two warps per 32-lane TMEM quarter (16 rows each), two
//               threads per row, one half of the block's keys each (the 16x32bx2 TMEM access
//               shape). A thread loads its 32 scores and a 48-column slice of its rows' BD'
//               window, hands S and BD' back at once (the next block's UMMAs overlap this
//               block's exponentials), applies the rel-shift BD[i][j] = BD'[i][j - i + 127] as a
//               per-lane shift of 0-15 by a 4-stage select network, takes the row maximum with one
//               shuffle, and writes its probabilities back to TMEM as f16 pairs.
// Lagging maximum (the TMEM accumulator is rescaled only when a row maximum grows by more than
// 2^8), 6 in 16 exponentials on the FMA pipe, paired f32 arithmetic, as the plain kernel
// (attention_fa.cu). Keys past a segment's length are masked; query rows past it are computed and
// not stored. Epilogue: the softmax warps read O from TMEM at once (the next item's first P·V may
// then overwrite it), normalise, stage their 16 rows each in the position slot of the item's last
// block and store them with one TMA box per warp; the producer refills that slot only after the
// stores have read it.
#include "kernels.cuh"
#include "ptx.cuh"
#include "softmax.cuh"

namespace wv {
namespace {

constexpr int BM = 128;                  // queries per CTA
constexpr int BN = 64;                   // keys per block
constexpr int HD = 128;                  // head size (the relative path's)
constexpr int PW_ROWS = BM + BN;         // position rows per block (191 used)
constexpr int SOFT_WARPS = 8;
constexpr int CTRL_WARPS = 3;            // TMA producer, S issuer, P·V issuer
constexpr int kRelPoly = 6;              // exponentials of 16 on the FMA pipe
constexpr int THREADS = 32 * (CTRL_WARPS + SOFT_WARPS);
constexpr int KVS = 2;                   // K / V ring slots
constexpr int PWS = 2;                   // position window slots

constexpr int ATOM_Q = BM * 128;         // one 64-column block of a 128-row tile
constexpr int ATOM_KV = BN * 128;
constexpr int ATOM_PW = PW_ROWS * 128;
constexpr int Q_BYTES = BM * HD * 2;
constexpr int KV_BYTES = BN * HD * 2;
constexpr int PW_BYTES = PW_ROWS * HD * 2;
constexpr int OFF_Q = 0;
constexpr int OFF_QV = OFF_Q + Q_BYTES;
constexpr int OFF_K = OFF_QV + Q_BYTES;
constexpr int OFF_V = OFF_K + KVS * KV_BYTES;
constexpr int OFF_PW = OFF_V + KVS * KV_BYTES;
constexpr int OFF_BAR = OFF_PW + PWS * PW_BYTES;
static_assert(SOFT_WARPS * 16 * HD * 2 <= 2 * KVS * KV_BYTES, "output staging (K and V rings)");
// TMEM columns: S (64 f32), BD' (192 f32), P (64 keys as f16 pairs), O (128 f32).
constexpr int T_S = 0;
constexpr int T_BD = 64;
constexpr int T_P = 256;
constexpr int T_O = 384;
constexpr int TMEM_COLS = 512;
constexpr uint32_t IDESC_S = idesc_f16(BM, BN, 0);
constexpr uint32_t IDESC_BD = idesc_f16(BM, PW_ROWS, 0);
constexpr uint32_t IDESC_PV = idesc_f16(BM, HD, 1);

struct __align__(8) RelBarriers {
  uint64_t q_full, q_empty;
  uint64_t k_full[KVS], k_empty[KVS];
  uint64_t v_full[KVS], v_empty[KVS];
  uint64_t pw_full[PWS], pw_empty[PWS];
  uint64_t s_full, s_free;
  uint64_t p_full, pv_done;
  uint64_t o_full, o_free;
  uint64_t stage_free[PWS];  // an item's output staging (in a position slot) has been stored
  uint64_t drain[2];
  uint32_t tmem_base;
  uint32_t abort;
};

// w[x] <- w[x + s] for x < 32, s in [0, 15], with static register indices (a select per element and
// stage; each stage makes just the outputs the later stages read).
template <int SH, int OUT>
__device__ __forceinline__ void shift_stage(float (&w)[48], bool take) {
#pragma unroll
  for (int x = 0; x < OUT; ++x) w[x] = take ? w[x + SH] : w[x];
}

__device__ __forceinline__ void shift_left16(float (&w)[48], uint32_t s) {
  shift_stage<8, 39>(w, (s >> 3) & 1u);
  shift_stage<4, 35>(w, (s >> 2) & 1u);
  shift_stage<2, 33>(w, (s >> 1) & 1u);
  shift_stage<1, 32>(w, s & 1u);
}

// One work item: 128 queries (tile x) of head h of segment seg.
struct RelItem {
  int h, m0, T, row0, nb;
};

// The CTA's items, the same sequence in every role: virtual items v = blockIdx.x + k·gridDim.x
// over (tile, head, segment), tile fastest; tiles that start past their segment are skipped.
struct RelItems {
  long long v, total;
  int ntiles;
  __device__ __forceinline__ bool next(const AttnArgs &a, RelItem &it) {
    while (v < total) {
      const int x = int(v % ntiles);
      const long long r = v / ntiles;
      const int h = int(r % a.heads), seg = int(r / a.heads);
      v += gridDim.x;
      const int T = a.seg_len ? a.seg_len[seg] : a.single_t;
      if (x * BM < T) {
        it.h = h;
        it.m0 = x * BM;
        it.T = T;
        it.row0 = a.seg_len ? a.seg_start[seg] : 0;
        it.nb = (T + BN - 1) / BN;
        return true;
      }
    }
    return false;
  }
};

__global__ void __launch_bounds__(THREADS, 1)
    rel_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_kv,
               const __grid_constant__ CUtensorMap map_pos,
               const __grid_constant__ CUtensorMap map_o, const AttnArgs a, int ntiles, int nseg) {
  const long long total = (long long)ntiles * a.heads * nseg;
  if (blockIdx.x >= total) return;  // uniform: the whole CTA leaves before any setup

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  RelBarriers *bar = reinterpret_cast<RelBarriers *>(smem + OFF_BAR);
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    mbar_init(&bar->q_empty, 1);
    for (int i = 0; i < KVS; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], 1);
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
    }
    for (int i = 0; i < PWS; ++i) {
      mbar_init(&bar->pw_full[i], 1);
      mbar_init(&bar->pw_empty[i], 1);
      mbar_init(&bar->stage_free[i], SOFT_WARPS);
    }
    mbar_init(&bar->s_full, 1);
    mbar_init(&bar->s_free, SOFT_WARPS);
    mbar_init(&bar->p_full, SOFT_WARPS);
    mbar_init(&bar->pv_done, 1);
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->o_free, SOFT_WARPS);
    mbar_init(&bar->drain[0], 1);
    mbar_init(&bar->drain[1], 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_kv);
    prefetch_tmap(&map_pos);
    if (a.o_tma) prefetch_tmap(&map_o);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, a.err};
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  RelItems items{blockIdx.x, total, ntiles};
  RelItem it;

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      uint32_t k_last[KVS] = {}, v_last[KVS] = {}, p_last[PWS] = {};  // bit 1: armed; 0: parity
      uint32_t q_last = 0;
      bool stage_pending[PWS] = {};
      uint32_t stage_waits[PWS] = {};
      uint32_t g = 0;  // key blocks of this CTA so far (ring slots and phases)
      for (uint32_t n = 0; ok && items.next(a, it); ++n) {
        const int hoff = it.h * a.head_stride;
        // Q and Q+v of this item once the previous item's last scores have read them.
        if (n > 0 && !mbar_wait(&bar->q_empty, (n - 1) & 1, ab, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bar->q_full, 2 * Q_BYTES);
        // 3D maps {64, rows, columns / 64}: one box holds a head's two 64-column chunks.
        tma_load_3d(smem + OFF_Q, &map_q, &bar->q_full, 0, it.row0 + it.m0, (a.q_off + hoff) / 64);
        tma_load_3d(smem + OFF_QV, &map_q, &bar->q_full, 0, it.row0 + it.m0,
                    (a.qv_off + hoff) / 64);
        q_last = 2u | (n & 1u);
        for (int j = 0; j < it.nb; ++j, ++g) {
          const uint32_t s = g % KVS, ps = g % PWS;
          const uint32_t par = ((g / KVS) & 1) ^ 1u, ppar = ((g / PWS) & 1) ^ 1u;
          if (!mbar_wait(&bar->k_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->k_full[s], KV_BYTES);
          tma_load_3d(smem + OFF_K + s * KV_BYTES, &map_kv, &bar->k_full[s], 0,
                      it.row0 + j * BN, (a.k_off + hoff) / 64);
          k_last[s] = 2u | ((g / KVS) & 1u);
          // A position slot that staged an earlier item's output is reused once that output has
          // been stored.
          if (stage_pending[ps]) {
            if (!mbar_wait(&bar->stage_free[ps], stage_waits[ps] & 1, ab, kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            ++stage_waits[ps];
            stage_pending[ps] = false;
          }
          if (!mbar_wait(&bar->pw_empty[ps], ppar, ab, kErrTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->pw_full[ps], PW_BYTES);
          // Position rows of block j: row r is relative position pos_t + 15 - r; the window
          // starts at the row of the largest i - j.
          const int rho0 = a.pos_t + 15 + j * BN - it.m0 - (BM - 1);
          tma_load_3d(smem + OFF_PW + ps * PW_BYTES, &map_pos, &bar->pw_full[ps], 0, rho0,
                      (a.pos_off + hoff) / 64);
          p_last[ps] = 2u | ((g / PWS) & 1u);
          if (!mbar_wait(&bar->v_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->v_full[s], KV_BYTES);
          tma_load_3d(smem + OFF_V + s * KV_BYTES, &map_kv, &bar->v_full[s], 0,
                      it.row0 + j * BN, (a.v_off + hoff) / 64);
          v_last[s] = 2u | ((g / KVS) & 1u);
        }
        if (ok) stage_pending[(g - 1) % PWS] = true;  // the item's output goes through this slot
      }
      if (!ok) {
        const long long t0 = clock64();
        auto drain = [&](uint64_t *b, uint32_t last) {
          if (!(last & 2u)) return;
          while (!mbar_try_wait(b, last & 1u) && clock64() - t0 < kWaitCycles) {
          }
        };
        drain(&bar->q_full, q_last);
        for (int s = 0; s < KVS; ++s) {
          drain(&bar->k_full[s], k_last[s]);
          drain(&bar->v_full[s], v_last[s]);
        }
        for (int s = 0; s < PWS; ++s) drain(&bar->pw_full[s], p_last[s]);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ---- UMMA issuers: warp 1 the scores (BD'(j), AC(j) as soon as the softmax holds block
    // j - 1's S and BD' in registers), warp 2 the accumulator (P(j)·V(j) once P(j) is in TMEM;
    // an item's first P·V once the softmax has read the previous item's O). A tcgen05.mma blocks
    // its thread while the tensor core is busy, so with one thread per stream one thread's
    // barrier waits overlap the other's UMMAs.
    if (lane == 0) {
      const bool is_s = warp == 1;
      bool ok = true;
      bool issued = false;
      // Descriptors are linear in the start address (bits 0-13 hold address / 16). Heads are 128
      // wide on this path (the host zero-pads narrower ones), so the score loops issue all eight
      // K-steps, unrolled and unconditional: issue loops with a guard on each UMMA produced wrong
      // scores, the unguarded and the rolled forms are exact.
      const uint64_t dq = sdesc_sw128(smem_u32(smem + OFF_Q), 16, 1024);
      const uint64_t dqv = sdesc_sw128(smem_u32(smem + OFF_QV), 16, 1024);
      const uint64_t dk = sdesc_sw128(smem_u32(smem + OFF_K), 16, 1024);
      const uint64_t dpw = sdesc_sw128(smem_u32(smem + OFF_PW), 16, 1024);
      const uint64_t dv = sdesc_sw128(smem_u32(smem + OFF_V), ATOM_KV, 1024);
      uint32_t g = 0;
      for (uint32_t n = 0; ok && items.next(a, it); ++n) {
        if (is_s && !mbar_wait(&bar->q_full, n & 1, ab, kErrTimeoutMma)) { ok = false; break; }
        for (int j = 0; j < it.nb; ++j, ++g) {
          if (is_s) {
            const uint32_t s = g % KVS, ps = g % PWS;
            if (!mbar_wait(&bar->k_full[s], (g / KVS) & 1, ab, kErrTimeoutMma) ||
                !mbar_wait(&bar->pw_full[ps], (g / PWS) & 1, ab, kErrTimeoutMma) ||
                (g >= 1 && !mbar_wait(&bar->s_free, (g - 1) & 1, ab, kErrTimeoutMma))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t bpw = dpw + uint64_t((ps * PW_BYTES) >> 4);
            const uint64_t bk = dk + uint64_t((s * KV_BYTES) >> 4);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint64_t oq = uint64_t(((kk >> 2) * ATOM_Q + (kk & 3) * 32) >> 4);
              umma_f16(tmem + T_BD, dqv + oq,
                       bpw + uint64_t(((kk >> 2) * ATOM_PW + (kk & 3) * 32) >> 4), IDESC_BD,
                       kk > 0 ? 1u : 0u);
            }
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint64_t oq = uint64_t(((kk >> 2) * ATOM_Q + (kk & 3) * 32) >> 4);
              umma_f16(tmem + T_S, dq + oq,
                       bk + uint64_t(((kk >> 2) * ATOM_KV + (kk & 3) * 32) >> 4), IDESC_S,
                       kk > 0 ? 1u : 0u);
            }
            issued = true;
            umma_commit(&bar->s_full);
            umma_commit(&bar->k_empty[s]);
            umma_commit(&bar->pw_empty[ps]);
          } else {
            const uint32_t vs = g % KVS;
            if (!mbar_wait(&bar->v_full[vs], (g / KVS) & 1, ab, kErrTimeoutMma) ||
                !mbar_wait(&bar->p_full, g & 1, ab, kErrTimeoutMma) ||
                (j == 0 && n > 0 && !mbar_wait(&bar->o_free, (n - 1) & 1, ab, kErrTimeoutMma))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t bv = dv + uint64_t((vs * KV_BYTES) >> 4);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              // A = P from TMEM: keys 16kk.. are columns 8kk.. of the P region; B = V rows 16kk..
              umma_f16_ts(tmem + T_O, tmem + T_P + kk * 8, bv + uint64_t((kk * 16 * 128) >> 4),
                          IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
            }
            issued = true;
            umma_commit(&bar->pv_done);
            umma_commit(&bar->v_empty[vs]);
          }
        }
        if (!ok) break;
        // The item's Q and Q+v may be replaced once its last scores completed; its O is final
        // once its last P·V completed.
        umma_commit(is_s ? &bar->q_empty : &bar->o_full);
      }
      if (!ok && issued) {
        uint64_t *dr = &bar->drain[is_s ? 0 : 1];
        umma_commit(dr);
        const long long t0 = clock64();
        while (!mbar_try_wait(dr, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ---- softmax: warps 3..10; rows r0 + (lane % 16), key half lane / 16 ----------------------
    const int w = int(warp) - CTRL_WARPS;
    const uint32_t quarter = warp & 3u;
    const int sub = w >> 2;
    const int ch = int(lane >> 4), d = int(lane & 15u);
    const int r0 = int(quarter) * 32 + sub * 16;
    const uint32_t tl = tmem + (uint32_t(r0) << 16);
    // BD' column of the first key of this thread's half, before its row's shift of 15 - d.
    const uint32_t bd0 = uint32_t(T_BD + (BM - 1) - r0 - 15);
    const float c = a.scale_log2;
    bool ok = true;
    uint32_t g = 0;
    for (uint32_t n = 0; ok && items.next(a, it); ++n) {
      const int T = it.T;
      float m_use = -INFINITY, l0 = 0.0f, l1 = 0.0f;
      for (int j = 0; j < it.nb; ++j, ++g) {
        if (!mbar_wait_warp(&bar->s_full, g & 1, ab, kErrTimeoutConsumer)) { ok = false; break; }
        tc_fence_after();
        float sc[32], bw[48];
        {
          uint32_t r[32], q0[16], q1[16], q2[16];
          tmem_ld_16x2_x32<32>(tl + T_S, r);
          tmem_ld_16x2_x16<32>(tl + bd0, q0);
          tmem_ld_16x2_x16<32>(tl + bd0 + 16, q1);
          tmem_ld_16x2_x16<32>(tl + bd0 + 32, q2);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) sc[x] = __uint_as_float(r[x]);
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            bw[x] = __uint_as_float(q0[x]);
            bw[16 + x] = __uint_as_float(q1[x]);
            bw[32 + x] = __uint_as_float(q2[x]);
          }
        }
        // S and BD' are in registers: the issuer may overwrite them with the next block's.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->s_free);
        shift_left16(bw, uint32_t(15 - d));
#pragma unroll
        for (int x = 0; x < 32; x += 2) add2(sc[x], sc[x + 1], sc[x], sc[x + 1], bw[x], bw[x + 1]);
        // Keys past the segment (last block only) are masked to -inf.
        const int kvalid = T - j * BN - ch * 32;
        if (kvalid < 32) {
#pragma unroll
          for (int x = 0; x < 32; ++x)
            if (x >= kvalid) sc[x] = -INFINITY;
        }
        float mx;
        {
          float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            float &m = m4[(x / 8) & 3];
            m = max3(m, sc[x + 0], sc[x + 1]);
            m = max3(m, sc[x + 2], sc[x + 3]);
            m = max3(m, sc[x + 4], sc[x + 5]);
            m = max3(m, sc[x + 6], sc[x + 7]);
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
        uint32_t pk[16];
#pragma unroll
        for (int gg = 0; gg < 32; gg += 16) {
          float *p = sc + gg;
#pragma unroll
          for (int x = 0; x < 16; x += 2) fma2(p[x], p[x + 1], p[x], p[x + 1], c, c, nm, nm);
          exp2_16<kRelPoly>(p);
#pragma unroll
          for (int x = 0; x < 16; x += 4) {
            float a0, a1;
            add2(a0, a1, p[x], p[x + 1], p[x + 2], p[x + 3]);
            add2(l0, l1, l0, l1, a0, a1);
          }
#pragma unroll
          for (int x = 0; x < 8; ++x) pk[gg / 2 + x] = pack_half2(p[2 * x], p[2 * x + 1]);
        }
        // P is free (and O stable) once the previous block's P·V landed, this item's or the last.
        if (g >= 1 && !mbar_wait_warp(&bar->pv_done, (g - 1) & 1, ab, kErrTimeoutConsumer)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_16x2_x16<16>(tl + T_P, pk);
        if (rescale) {
#pragma unroll 1
          for (int q = 0; q < HD / 2 / 16; ++q) {
            uint32_t r[16];
            tmem_ld_16x2_x16<HD / 2>(tl + T_O + q * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 16; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * alpha);
            tmem_st_16x2_x16<HD / 2>(tl + T_O + q * 16, r);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->p_full);
      }
      if (!ok || !mbar_wait_warp(&bar->o_full, n & 1, ab, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      // ---- epilogue: this thread's half of its row of O, read at once so that the next item's
      // first P·V may overwrite the accumulator while the rows are normalised and stored.
      tc_fence_after();
      uint32_t ov[HD / 2];
      tmem_ld_16x2_x32<HD / 2>(tl + T_O, *reinterpret_cast<uint32_t(*)[32]>(ov));
      tmem_ld_16x2_x32<HD / 2>(tl + T_O + 32, *reinterpret_cast<uint32_t(*)[32]>(ov + 32));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->o_free);
      // The row sum over both halves.
      float l = l0 + l1;
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      const float inv = 1.0f / l;
      const int m0 = it.m0, hd = a.hd;
      const int qrow = m0 + r0 + d;
      const bool store = qrow < T;
      // A warp whose 16 rows all lie in the segment stages them in the position slot of the
      // item's last block (read by its last scores; the producer reuses the slot only after
      // stage_free) and stores them with one TMA box; a partial group is stored row by row.
      const uint32_t slot = (g - 1) % PWS;
      const bool via_tma = a.o_tma && m0 + r0 + 16 <= T;
      uint8_t *stage_w = smem + OFF_PW + slot * PW_BYTES + w * (16 * HD * 2);
      uint8_t *stage = stage_w + d * (hd * 2);
      const long long orow = (long long)(it.row0 + qrow) * a.ldo + (long long)it.h * hd;
#pragma unroll
      for (int q = 0; q < HD / 2 / 32; ++q) {
        const uint32_t *r = ov + q * 32;
        const int c0 = ch * (HD / 2) + q * 32;
        if (via_tma) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            if (c0 + x < hd) {  // the head size is a multiple of 8 on this path
              const uint4 v = make_uint4(
                  pack_half2(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv),
                  pack_half2(__uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv),
                  pack_half2(__uint_as_float(r[x + 4]) * inv, __uint_as_float(r[x + 5]) * inv),
                  pack_half2(__uint_as_float(r[x + 6]) * inv, __uint_as_float(r[x + 7]) * inv));
              *reinterpret_cast<uint4 *>(stage + (c0 + x) * 2) = v;
            }
          }
        } else if (store && c0 < hd) {
          if (a.o_f16) {
            __half *o = reinterpret_cast<__half *>(a.o) + orow;
            if (c0 + 32 <= hd && ((reinterpret_cast<uintptr_t>(o + c0) & 15u) == 0)) {
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
                if (c0 + x < hd) o[c0 + x] = __float2half_rn(__uint_as_float(r[x]) * inv);
            }
          } else {
            float *o = reinterpret_cast<float *>(a.o) + orow;
#pragma unroll
            for (int x = 0; x < 32; ++x)
              if (c0 + x < hd) o[c0 + x] = __uint_as_float(r[x]) * inv;
          }
        }
      }
      if (via_tma) {
        fence_proxy_async_smem();  // the staged rows are visible to the TMA (async proxy)
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_o, stage_w, it.h * hd, it.row0 + m0 + r0);
          bulk_commit();
          // The slot may be refilled once the TMA has read it; the writes complete with the grid.
          bulk_wait_read<0>();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->stage_free[slot]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// f32 or f16 operand rows -> f16 rows with heads padded to hd_pad.
__global__ void pack_heads_kernel(const void *__restrict__ in, int in_f16, long long ld_in,
                                  const int4 offs, int sections, __half *__restrict__ out,
                                  long long ld_out, int rows, int heads, int hd, int hd_pad) {
  const long long width = (long long)sections * heads * hd_pad;
  for (long long row = blockIdx.y; row < rows; row += gridDim.y) {
    for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < width;
         c += (long long)gridDim.x * blockDim.x) {
      const int sec = int(c / (heads * hd_pad));
      const int rem = int(c % (heads * hd_pad));
      const int hh = rem / hd_pad, x = rem % hd_pad;
      const int off = sec == 0 ? offs.x : sec == 1 ? offs.y : sec == 2 ? offs.z : offs.w;
      float v = 0.0f;
      if (x < hd) {
        const long long at = row * ld_in + off + (long long)hh * hd + x;
        v = in_f16 ? __half2float(reinterpret_cast<const __half *>(in)[at])
                   : reinterpret_cast<const float *>(in)[at];
      }
      out[row * ld_out + c] = __float2half_rn(v);
    }
  }
}

cudaError_t launch_rel(const CUtensorMap &q, const CUtensorMap &kv, const CUtensorMap &pos,
                       const CUtensorMap &o, const AttnArgs &a, int max_len, int nseg,
                       cudaStream_t s) {
  const size_t smem = 1024 + OFF_BAR + sizeof(RelBarriers);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(rel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  // Persistent: one CTA per SM (224 KB of shared memory and all of TMEM each) walks its items.
  static int sms[64] = {};
  if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int ntiles = (max_len + BM - 1) / BM;
  const long long items = (long long)ntiles * a.heads * nseg;
  const int nsm = dev < 64 && sms[dev] > 0 ? sms[dev] : 148;
  const int grid = int(items < nsm ? items : nsm);
  return launch_pdl(rel_kernel, dim3(grid), dim3(THREADS), smem, s, q, kv, pos, o, a, ntiles, nseg);
}

}  // namespace

cudaError_t launch_attention(const CUtensorMap &map_q, const CUtensorMap &map_kv,
                             const CUtensorMap &map_pos, const CUtensorMap &map_o,
                             const AttnArgs &a, int hd_pad, bool rel, int max_len, int nseg,
                             cudaStream_t s) {
  if (max_len <= 0 || nseg <= 0) return cudaSuccess;
  if (rel) return launch_rel(map_q, map_kv, map_pos, map_o, a, max_len, nseg, s);
  return launch_fa_attention(map_q, map_kv, map_o, a, hd_pad, max_len, nseg, s);
}

int attn_block_keys(bool rel, int hd_pad) { return rel ? BN : fa_block_keys(hd_pad); }
int attn_pos_window_rows() { return PW_ROWS; }

cudaError_t launch_pack_heads(const void *in, int in_f16, long long ld_in, const int *in_off,
                              int sections, __half *out, long long ld_out, int rows, int heads,
                              int hd, int hd_pad, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  int4 offs = make_int4(in_off[0], sections > 1 ? in_off[1] : 0, sections > 2 ? in_off[2] : 0,
                        sections > 3 ? in_off[3] : 0);
  const long long width = (long long)sections * heads * hd_pad;
  int bx = int((width + 255) / 256);
  if (bx > 32) bx = 32;
  dim3 grid(bx, rows < 65535 ? rows : 65535);
  pack_heads_kernel<<<grid, 256, 0, s>>>(in, in_f16, ld_in, offs, sections, out, ld_out, rows,
                                         heads, hd, hd_pad);
  return cudaGetLastError();
}

}  // namespace wv
