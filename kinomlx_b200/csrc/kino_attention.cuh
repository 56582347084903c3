// Dense attention on tcgen05 for 128- or 64-wide heads (template D), bf16 in and out, fp32
// softmax/accumulation.
//
// Restates the math of the reference's attention calls: softmax(q k^T * d^-1/2) v per head
// (kinomlx/models/flux2/kv.py:48-54 joint attention through MLX SDPA,
//  kinomlx/models/ltx2/kernels/dense_attention.py:107-151 token-major dense attention,
//  kinomlx/models/ltx2/transformer/attention.py:144-161 unmasked SDPA, 364-368 head gates).
//
// Layout: q, k and v are token-major, (batch, tokens, heads * D) with any row stride, which is
// what the projections write. Queries and keys may each come in two segments (text tokens, then
// image tokens) that are concatenated logically but never in memory: each 128-row query tile and
// each 128-key block belongs to one segment.
//
// One CTA computes two 128-query tiles (A and B) of one head in ping-pong:
//   warp 0      TMA: Q_A and Q_B once, then K and V blocks of 128 keys through a 2-stage ring
//   warp 1      tensor-memory owner and MMA issuer, in the order
//                 S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) | ...
//               so one tile's products run while the other tile's softmax does
//   warps 2..9  the softmax of whichever tile is next, A(j), B(j), A(j+1), ...: two warps per
//               tensor-memory lane quarter (32 query rows), each on 64 of the block's 128 keys;
//               tcgen05.ld the half row, exchange the half-row maxima through shared memory (an
//               mbarrier per quarter), exponentials in the exp2 domain (part on the FMA pipes),
//               P as bf16 pairs back over the half's own scores. O is rescaled in tensor memory
//               only when the running max grows by more than 2^8 (the stale max cancels in the
//               final division).
// Tensor memory (512 columns): S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [384,384+D). P of
// keys 0..63 sits in columns [0,32) and of keys 64..127 in [64,96) of its S. The PV product takes
// P straight from tensor memory (the TMEM-A form of tcgen05.mma) and V in place from shared
// memory as an MN-major operand. MMAs of one issuing thread run in order, so S(j+1) overwriting
// P(j) after PV(j) is safe, and the commit that signals S(j+1) also covers PV(j), so O is
// settled whenever the softmax sees S.
#pragma once
#include "kino_common.cuh"

namespace kino {

constexpr int ATT_BM = 128;  // queries per tile
constexpr int ATT_BN = 128;  // keys per block
constexpr int ATT_D = 128;   // widest head dim (the shared-memory layout holds 128)
constexpr int ATT_STAGES = 2;  // K + V blocks in flight
constexpr int ATT_THREADS = 320;
// Key pairs i of a block whose bit (i % 8) is set take the FMA-pipe exponential
// (exp2_poly_x2) instead of the special-function unit: bits 1, 4, 6 = 3 of every 8 pairs.
#ifndef KINO_ATT_EMU_MASK
#define KINO_ATT_EMU_MASK 0x52
#endif
constexpr unsigned ATT_EMU_MASK = KINO_ATT_EMU_MASK;

struct AttnParams {
  int batch, heads;
  int nq_seg, nkv_seg;
  int q_tokens[2], q_tiles[2];
  int kv_tokens[2], kv_blocks[2];
  __nv_bfloat16* out[2];
  int64_t ld_out[2], bs_out[2];
  const __nv_bfloat16* gate[2];  // optional (batch, tokens, heads) output gate per query segment
  int64_t ld_gate[2], bs_gate[2];
  float scale_log2;
  // Sequence-parallel return (batch 1, one query segment): query row t belongs to rank
  // t / rows_per_rank; its output goes to out_peers[rank] + (t % rows_per_rank) * ld_out[0] +
  // out_col_offset + head * 128 and its gate is read from gate_peers[rank] (row stride
  // ld_gate[0], column gate_head_offset + head). Null out_peers: plain `out`.
  __nv_bfloat16* const* out_peers;
  const __nv_bfloat16* const* gate_peers;
  int rows_per_rank;
  int64_t out_col_offset;
  int gate_head_offset;
  // Optional additive key bias (the BIAS instantiation, one key segment): key_bias[batch *
  // ld_key_bias + key] is added to q k^T * scale (natural-log units), as an additive attention
  // mask is (kinomlx/models/ltx2/transformer/attention.py:164-186).
  const float* key_bias;
  int64_t ld_key_bias;
  // Split keys (kv_splits > 1, no key bias): CTA x covers tile pair x / kv_splits and the
  // kv_splits-th share x % kv_splits of the key blocks, and writes its unnormalised output and
  // row statistics instead of `out`: part_o[((split * batch + b) * heads + h) * rows + r][D]
  // (fp32; r = global tile index * 128 + row over both query segments) and part_ml[...][2]
  // (row maximum in log2 units, row sum); attention_combine_kernel merges the shares.
  int kv_splits;
  int64_t part_rows;
  float* part_o;
  float* part_ml;
};

struct AttnSmem {
  static constexpr int HALF = 128 * 64 * 2;    // 16 KB: 128 rows x 64 dims
  static constexpr int Q_OFF = 0;              // tile t at Q_OFF + t * 2 * HALF
  static constexpr int KV_OFF = 4 * HALF;      // per stage: K 2 halves, V 2 halves
  static constexpr int STAGE = 4 * HALF;
  static constexpr int X_OFF = KV_OFF + ATT_STAGES * STAGE;  // maxima [tile][parity][half][128]
  static constexpr int L_OFF = X_OFF + 2 * 2 * 2 * 128 * 4;  // sums [tile][half][128]
  static constexpr int BAR_OFF = L_OFF + 2 * 2 * 128 * 4;
  // q_full, kv_full[S], kv_empty[S], s_full[2], p_full[2], o_done, drain, xbar[4][2][2], lbar[4]
  static constexpr int NBAR = 1 + 2 * ATT_STAGES + 2 + 2 + 2 + 16 + 4;
  static constexpr int TOTAL = BAR_OFF + NBAR * 8 + 16 + 1024;
};

// MN-major 128-byte-swizzled operand: 64 contiguous MN elements per 128-byte row, rows along K
// 128 bytes apart, 8-row groups 1024 bytes apart (SBO), 64-element MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// D (tensor memory) += A (tensor memory, 128 lanes x 16 bf16 packed in 8 columns) * B (smem).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

struct QTile {
  int seg, tile;
  bool valid;
};

__device__ __forceinline__ QTile q_tile_of(const AttnParams& p, int global) {
  QTile t;
  const int total = p.q_tiles[0] + (p.nq_seg > 1 ? p.q_tiles[1] : 0);
  t.valid = global < total;
  t.seg = (global < p.q_tiles[0]) ? 0 : 1;
  t.tile = global - (t.seg ? p.q_tiles[0] : 0);
  return t;
}

template <int D, bool BIAS = false, bool SPLIT = false>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap mq0,
                        const __grid_constant__ CUtensorMap mq1,
                        const __grid_constant__ CUtensorMap mk0,
                        const __grid_constant__ CUtensorMap mk1,
                        const __grid_constant__ CUtensorMap mv0,
                        const __grid_constant__ CUtensorMap mv1, const AttnParams p) {
  using L = AttnSmem;
  static_assert(D == 64 || D == 128, "heads are 64 or 128 wide");
  constexpr int NH = D / 64;  // 64-wide halves of a head (one 128-byte swizzle row each)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ATT_STAGES;
  uint64_t* s_full = kv_empty + ATT_STAGES;  // [tile]
  uint64_t* p_full = s_full + 2;             // [tile]
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 1;
  uint64_t* xbar = drain + 1;                // [quarter][tile][block parity]
  uint64_t* lbar = xbar + 16;                // [quarter]
  float* xmax = reinterpret_cast<float*>(smem + L::X_OFF);
  float* xsum = reinterpret_cast<float*>(smem + L::L_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int splits = SPLIT ? p.kv_splits : 1;
  const int pair = blockIdx.x / splits, split = blockIdx.x % splits;
  const QTile tiles[2] = {q_tile_of(p, 2 * pair), q_tile_of(p, 2 * pair + 1)};
  const bool has_b = tiles[1].valid;
  const int ntile = has_b ? 2 : 1;
  // this CTA's key blocks [b0, b0 + nblk) of all segments' blocks
  const int nblk_all = p.kv_blocks[0] + (p.nkv_seg > 1 ? p.kv_blocks[1] : 0);
  const int b0 = split * nblk_all / splits;
  const int nblk = (split + 1) * nblk_all / splits - b0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ATT_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 8);  // one arrive per softmax warp
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 16; ++i) mbar_init(&xbar[i], 64);  // the two warps of a quarter
    for (int i = 0; i < 4; ++i) mbar_init(&lbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  griddep_wait();  // the previous kernel has finished with its memory and tensor memory
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, (has_b ? 2 : 1) * NH * L::HALF);
      for (int t = 0; t < ntile; ++t) {
        const CUtensorMap* mq = tiles[t].seg ? &mq1 : &mq0;
        uint8_t* sq = smem + L::Q_OFF + t * 2 * L::HALF;
        tma_load_4d(sq, mq, q_full, 0, tiles[t].tile * ATT_BM, head, batch);
        if (NH > 1) tma_load_4d(sq + L::HALF, mq, q_full, 64, tiles[t].tile * ATT_BM, head, batch);
      }
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int stage = j % ATT_STAGES;
        const uint32_t parity = (j / ATT_STAGES) & 1;
        if (!mbar_wait(&kv_empty[stage], parity ^ 1u, abort_flag)) break;
        const int kseg = (b0 + j < p.kv_blocks[0]) ? 0 : 1;
        const int kb = b0 + j - (kseg ? p.kv_blocks[0] : 0);
        const CUtensorMap* mk = kseg ? &mk1 : &mk0;
        const CUtensorMap* mv = kseg ? &mv1 : &mv0;
        uint8_t* sk = smem + L::KV_OFF + stage * L::STAGE;
        uint8_t* sv = sk + 2 * L::HALF;
        mbar_expect_tx(&kv_full[stage], 2 * NH * L::HALF);
        const int t0 = kb * ATT_BN;
#pragma unroll
        for (int h2 = 0; h2 < NH; ++h2) {
          tma_load_4d(sk + h2 * L::HALF, mk, &kv_full[stage], h2 * 64, t0, head, batch);
          tma_load_4d(sv + h2 * L::HALF, mv, &kv_full[stage], h2 * 64, t0, head, batch);
        }
        ++issued;
      }
      if (*abort_flag) {
        // Let copies in flight land before the CTA retires (bounded).
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(q_full, 0) && global_ns() - t0 < 200000000ull) {
        }
        for (int j = issued - 1; j >= 0 && j >= issued - ATT_STAGES; --j) {
          const uint64_t t1 = global_ns();
          while (!mbar_try_wait(&kv_full[j % ATT_STAGES], (j / ATT_STAGES) & 1) &&
                 global_ns() - t1 < 200000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(ATT_BM, ATT_BN);
      constexpr uint32_t idesc_o = idesc_bf16(ATT_BM, D) | (1u << 16);  // B (V) MN-major
      auto s_mma = [&](int t, int j) {
        const uint32_t sq = smem_u32(smem + L::Q_OFF + t * 2 * L::HALF);
        const uint32_t sk = smem_u32(smem + L::KV_OFF + (j % ATT_STAGES) * L::STAGE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::HALF + (kk & 3) * 32;
          umma_bf16(tmem + t * 128, sdesc_k128(sq + off), sdesc_k128(sk + off), idesc_s,
                    kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto pv_mma = [&](int t, int j) {
        const uint32_t sv =
            smem_u32(smem + L::KV_OFF + (j % ATT_STAGES) * L::STAGE + 2 * L::HALF);
#pragma unroll
        for (int kk = 0; kk < ATT_BN / 16; ++kk) {
          // keys 16kk .. 16kk+15: P columns 8kk (first 64 keys) or 8kk + 32 (last 64)
          umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8 + (kk >= 4 ? 32 : 0),
                       sdesc_mn128(sv + kk * 2048, L::HALF), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, abort_flag) && nblk > 0;
      if (ok) ok = mbar_wait(&kv_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < ntile; ++t) s_mma(t, 0);
      }
      for (int j = 0; ok && j < nblk; ++j) {
        const bool more = j + 1 < nblk;
        for (int t = 0; t < ntile && ok; ++t) {
          if (!mbar_wait(&p_full[t], j & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          pv_mma(t, j);
          if (t == ntile - 1) umma_commit(&kv_empty[j % ATT_STAGES]);
          if (more) {
            if (t == 0) {
              if (!mbar_wait(&kv_full[(j + 1) % ATT_STAGES], ((j + 1) / ATT_STAGES) & 1,
                             abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            s_mma(t, j + 1);
          }
        }
      }
      umma_commit(o_done);
      umma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 200000000ull) {
      }
    }
  } else {
    // softmax warps 2..9: lane quarter warp % 4 (32 rows), key half (warp - 2) / 4
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + static_cast<int>(lane);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m_run[2] = {-INFINITY, -INFINITY};  // per tile: running max of s * scale * log2(e)
    float l_run[2] = {0.0f, 0.0f};            // per tile: this half's share of the row sum
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      const int kseg = (b0 + j < p.kv_blocks[0]) ? 0 : 1;
      const int kb = b0 + j - (kseg ? p.kv_blocks[0] : 0);
      const int valid = min(ATT_BN, p.kv_tokens[kseg] - kb * ATT_BN) - half * 64;
      // BIAS: this half block's key biases in log2 units, floored at -1e30 so that a row whose
      // keys are all masked averages them uniformly, as a finite additive mask does
      float kbias[BIAS ? 64 : 1];
      if constexpr (BIAS) {
        const float4* bp = reinterpret_cast<const float4*>(
            p.key_bias + static_cast<int64_t>(batch) * p.ld_key_bias + kb * ATT_BN + half * 64);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float4 b4 = c * 4 < valid ? bp[c] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          kbias[c * 4 + 0] = fmaxf(b4.x * 1.4426950408889634f, -1.0e30f);
          kbias[c * 4 + 1] = fmaxf(b4.y * 1.4426950408889634f, -1.0e30f);
          kbias[c * 4 + 2] = fmaxf(b4.z * 1.4426950408889634f, -1.0e30f);
          kbias[c * 4 + 3] = fmaxf(b4.w * 1.4426950408889634f, -1.0e30f);
        }
      }
      for (int t = 0; t < ntile; ++t) {
        if (!mbar_wait(&s_full[t], j & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_col = tmem + lane_base + t * 128 + half * 64;
        uint32_t sr[2][32];
        tmem_ld32(s_col, sr[0]);
        tmem_ld32(s_col + 32, sr[1]);
        tmem_wait_ld();
        if (valid < 64) {  // only a segment's last key block; warp-uniform
#pragma unroll
          for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i >= valid) sr[c][i] = __float_as_uint(-INFINITY);
          }
        }
        if constexpr (BIAS) {  // logits in log2 units from here on
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              sr[c][i] = __float_as_uint(fmaf(__uint_as_float(sr[c][i]), sl2, kbias[c * 32 + i]));
        }
        float mq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t* v = sr[q >> 1] + (q & 1) * 16;
          float a = max3f(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]));
          a = max3f(a, __uint_as_float(v[3]), __uint_as_float(v[4]));
          a = max3f(a, __uint_as_float(v[5]), __uint_as_float(v[6]));
          a = max3f(a, __uint_as_float(v[7]), __uint_as_float(v[8]));
          a = max3f(a, __uint_as_float(v[9]), __uint_as_float(v[10]));
          a = max3f(a, __uint_as_float(v[11]), __uint_as_float(v[12]));
          a = max3f(a, __uint_as_float(v[13]), __uint_as_float(v[14]));
          mq[q] = fmaxf(a, __uint_as_float(v[15]));
        }
        const float mine = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        // exchange the half-row maxima with the quarter's other warp
        float* xm = xmax + (t * 2 + (j & 1)) * 256;
        xm[half * 128 + row] = mine;
        uint64_t* xb = &xbar[(quarter * 2 + t) * 2 + (j & 1)];
        mbar_arrive(xb);
        if (!mbar_wait(xb, (j >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        const float m_blk = fmaxf(mine, xm[(1 - half) * 128 + row]) * (BIAS ? 1.0f : sl2);
        // Lazy rescale, decided identically by both halves of a row. O of this tile holds PV(j-1)
        // (completed before S(j) was signalled).
        float alpha = 1.0f;
        bool rescale = false;
        if (j > 0) {
          const bool need = m_blk > m_run[t] + 8.0f;
          rescale = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = ex2_approx(m_run[t] - m_blk);
            m_run[t] = m_blk;
            l_run[t] *= alpha;
          }
        } else {
          m_run[t] = m_blk;
        }
        const float mult = BIAS ? 1.0f : sl2;
        const uint64_t sl2x2 = f2_pack(mult, mult);
        const uint64_t negm = f2_pack(-m_run[t], -m_run[t]);
        uint64_t lsum2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          uint32_t packed[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int i = q8 * 8 + u;  // key pair index within the half block
            const uint32_t* v = sr[i >> 4];
            const int e = (2 * i) & 31;
            const uint64_t xs =
                f2_fma(f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sl2x2, negm);
            uint64_t ev;
            if ((ATT_EMU_MASK >> (i & 7)) & 1) {
              ev = exp2_poly_x2(xs);
            } else {
              const float2 xv = f2_unpack(xs);
              ev = f2_pack(ex2_approx(xv.x), ex2_approx(xv.y));
            }
            lsum2[u & 1] = f2_add(lsum2[u & 1], ev);
            const float2 e2 = f2_unpack(ev);
            packed[u] = pack_bf16x2(e2.x, e2.y);
          }
          tmem_st8(s_col + q8 * 8, packed);
        }
        const float2 ls = f2_unpack(f2_add(lsum2[0], lsum2[1]));
        l_run[t] += ls.x + ls.y;
        if (rescale) {
          const uint32_t o_col = tmem + lane_base + 256 + t * 128 + half * (D / 2);
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            tmem_ld32(o_col + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_col + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
    }
    if (ok && nblk > 0) {
      // row sums: this half's shares to shared memory for the other warp of the quarter
      for (int t = 0; t < ntile; ++t) xsum[(t * 2 + half) * 128 + row] = l_run[t];
      mbar_arrive(&lbar[quarter]);
      ok = mbar_wait(&lbar[quarter], 0, abort_flag);
    }
    if (SPLIT && ok && nblk > 0 && mbar_wait(o_done, 0, abort_flag)) {
      // one share of the keys: the unnormalised output and the row statistics
      tc_fence_after();
      for (int t = 0; t < ntile; ++t) {
        const QTile qt = tiles[t];
        const bool store = qt.tile * ATT_BM + row < p.q_tokens[qt.seg];
        const int64_t r = static_cast<int64_t>(2 * pair + t) * ATT_BM + row;
        const int64_t slot = ((static_cast<int64_t>(split) * p.batch + batch) * p.heads + head) *
                                 p.part_rows + r;
        if (store && half == 0) {
          p.part_ml[slot * 2] = m_run[t];
          p.part_ml[slot * 2 + 1] = l_run[t] + xsum[(t * 2 + 1) * 128 + row];
        }
        float* dst = p.part_o + slot * D + half * (D / 2);
        const uint32_t o_col = tmem + lane_base + 256 + t * 128 + half * (D / 2);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
          if (store) {
#pragma unroll
            for (int g = 0; g < 8; ++g)
              *reinterpret_cast<uint4*>(dst + c * 32 + g * 4) =
                  make_uint4(o[g * 4], o[g * 4 + 1], o[g * 4 + 2], o[g * 4 + 3]);
          }
        }
      }
    } else if (ok && nblk > 0 && mbar_wait(o_done, 0, abort_flag)) {
      tc_fence_after();
      for (int t = 0; t < ntile; ++t) {
        const QTile qt = tiles[t];
        const int tok = qt.tile * ATT_BM + row;
        const bool store = tok < p.q_tokens[qt.seg];
        const float inv_l = 1.0f / (l_run[t] + xsum[(t * 2 + 1 - half) * 128 + row]);
        // Optional head gate: bf16(bf16(O / l) * gate[t, head])
        const __nv_bfloat16* gp = p.gate[qt.seg];
        __nv_bfloat16* dst;
        float gv = 1.0f;
        if (p.out_peers != nullptr) {
          // the row's owner GPU: its output buffer and its gate, over NVLink
          const int owner = tok / p.rows_per_rank;
          const int64_t lt = tok - static_cast<int64_t>(owner) * p.rows_per_rank;
          dst = (store ? p.out_peers[owner] : p.out_peers[0]) + lt * p.ld_out[0] +
                p.out_col_offset + head * D;
          if (p.gate_peers != nullptr) {
            gp = p.gate_peers[0];
            if (store)
              gv = __bfloat162float(
                  p.gate_peers[owner][lt * p.ld_gate[0] + p.gate_head_offset + head]);
          }
        } else {
          dst = p.out[qt.seg] + static_cast<int64_t>(batch) * p.bs_out[qt.seg] +
                static_cast<int64_t>(tok) * p.ld_out[qt.seg] + head * D;
          if (gp != nullptr && store)
            gv = __bfloat162float(gp[static_cast<int64_t>(batch) * p.bs_gate[qt.seg] +
                                     static_cast<int64_t>(tok) * p.ld_gate[qt.seg] + head]);
        }
        auto fin = [&](uint32_t raw) -> float {
          const float o = __uint_as_float(raw) * inv_l;
          return gp != nullptr ? bf16_round(bf16_round(o) * gv) : o;
        };
        const uint32_t o_col = tmem + lane_base + 256 + t * 128 + half * (D / 2);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
          if (store) {
            uint32_t w16[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) w16[j] = pack_bf16x2(fin(o[2 * j]), fin(o[2 * j + 1]));
            store_row32(dst + half * (D / 2) + c * 32, w16, 32);
          }
        }
      }
      // rows returned to other GPUs: visible before the next kernel signals
      if (p.out_peers != nullptr) __threadfence_system();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Merge of the key shares of a split attention (AttnParams::kv_splits > 1): one thread per 8
// output columns of a (batch, head, query row): O = sum_i O_i 2^(m_i - m) / sum_i l_i 2^(m_i - m)
// over the shares i, then the one-pass kernel's gate and store (local rows, or the owner GPU's
// rows under the sequence-parallel return).
template <int D>
__global__ void __launch_bounds__(256) attention_combine_kernel(const AttnParams p) {
  griddep_wait();
  griddep_launch();
  constexpr int CH = D / 8;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  const int c = static_cast<int>(gid % CH);
  const int64_t r = (gid / CH) % p.part_rows;
  const int64_t bh = gid / (CH * p.part_rows);
  if (bh >= static_cast<int64_t>(p.batch) * p.heads) return;
  const int batch = static_cast<int>(bh / p.heads), head = static_cast<int>(bh % p.heads);
  const QTile qt = q_tile_of(p, static_cast<int>(r / ATT_BM));
  const int tok = qt.tile * ATT_BM + static_cast<int>(r % ATT_BM);
  if (!qt.valid || tok >= p.q_tokens[qt.seg]) return;
  const int64_t stride = static_cast<int64_t>(p.batch) * p.heads * p.part_rows;  // per share
  const int64_t slot0 = bh * p.part_rows + r;
  float m = -INFINITY;
  for (int i = 0; i < p.kv_splits; ++i) m = fmaxf(m, p.part_ml[(slot0 + i * stride) * 2]);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float l = 0.0f;
  for (int i = 0; i < p.kv_splits; ++i) {
    const int64_t slot = slot0 + i * stride;
    const float w = ex2_approx(p.part_ml[slot * 2] - m);
    l += p.part_ml[slot * 2 + 1] * w;
    const float4* src = reinterpret_cast<const float4*>(p.part_o + slot * D + c * 8);
    const float4 a = src[0], b = src[1];
    acc[0] += a.x * w;
    acc[1] += a.y * w;
    acc[2] += a.z * w;
    acc[3] += a.w * w;
    acc[4] += b.x * w;
    acc[5] += b.y * w;
    acc[6] += b.z * w;
    acc[7] += b.w * w;
  }
  const float inv_l = 1.0f / l;
  const __nv_bfloat16* gp = p.gate[qt.seg];
  __nv_bfloat16* dst;
  float gv = 1.0f;
  if (p.out_peers != nullptr) {
    const int owner = tok / p.rows_per_rank;
    const int64_t lt = tok - static_cast<int64_t>(owner) * p.rows_per_rank;
    dst = p.out_peers[owner] + lt * p.ld_out[0] + p.out_col_offset + head * D;
    if (p.gate_peers != nullptr) {
      gp = p.gate_peers[0];
      gv = __bfloat162float(p.gate_peers[owner][lt * p.ld_gate[0] + p.gate_head_offset + head]);
    }
  } else {
    dst = p.out[qt.seg] + static_cast<int64_t>(batch) * p.bs_out[qt.seg] +
          static_cast<int64_t>(tok) * p.ld_out[qt.seg] + head * D;
    if (gp != nullptr)
      gv = __bfloat162float(gp[static_cast<int64_t>(batch) * p.bs_gate[qt.seg] +
                               static_cast<int64_t>(tok) * p.ld_gate[qt.seg] + head]);
  }
  float o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    o[e] = acc[e] * inv_l;
    if (gp != nullptr) o[e] = bf16_round(bf16_round(o[e]) * gv);
  }
  *reinterpret_cast<uint4*>(dst + c * 8) =
      make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                 pack_bf16x2(o[6], o[7]));
  if (p.out_peers != nullptr) __threadfence_system();
}

}  // namespace kino
