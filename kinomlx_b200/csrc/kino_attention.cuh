// Dense attention on tcgen05 for 128-wide heads, bf16 in and out, fp32 softmax/accumulation.
//
// Restates the math of the reference's attention calls: softmax(q k^T * d^-1/2) v per head
// (kinomlx/models/flux2/kv.py:48-54 joint attention through MLX SDPA,
//  kinomlx/models/ltx2/kernels/dense_attention.py:107-151 token-major dense attention,
//  kinomlx/models/ltx2/transformer/attention.py:144-161 unmasked SDPA).
//
// Layout: q, k and v are token-major, (batch, tokens, heads * 128) with any row stride, which is
// what the projections write; the reference's dense kernel takes the same layout. Queries and
// keys may each come in two segments (text tokens, then image tokens) that are concatenated
// logically but never in memory: each 128-row tile belongs to one segment.
//
// One CTA computes 128 queries of one head:
//   warp 0      TMA: Q once, then K and V tiles of 128 keys through a 2-stage ring
//   warp 1      tensor memory owner and MMA issuer: S = Q K^T into one of two S buffers,
//               O += P V into the O buffer
//   warps 2..5  softmax, one query row per thread: tcgen05.ld the S row, online max/sum in the
//               exp2 domain, rescale O in tensor memory only when the running max grows by more
//               than 2^8 (exact: the stale max cancels in the final division), write P as bf16
//               into 128-byte-swizzled shared memory for the next MMA, finally O / l.
// V is consumed in place as an MN-major operand (no transpose pass).
#pragma once
#include "kino_common.cuh"

namespace kino {

constexpr int ATT_BM = 128;       // queries per CTA
constexpr int ATT_BN = 128;       // keys per block
constexpr int ATT_D = 128;        // head dim
constexpr int ATT_STAGES = 2;
constexpr int ATT_THREADS = 192;

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
};

struct AttnSmem {
  static constexpr int HALF = ATT_BM * 64 * 2;             // 16 KB: 128 rows x 128 bytes
  static constexpr int Q_OFF = 0;                          // 2 halves (d 0..63, 64..127)
  static constexpr int P_OFF = Q_OFF + 2 * HALF;           // 2 halves (keys 0..63, 64..127)
  static constexpr int KV_OFF = P_OFF + 2 * HALF;          // per stage: K 2 halves, V 2 halves
  static constexpr int STAGE = 4 * HALF;
  static constexpr int BAR_OFF = KV_OFF + ATT_STAGES * STAGE;
  // q_full, kv_full[S], kv_empty[S], s_full[2], p_full, o_done, drain
  static constexpr int NBAR = 1 + 2 * ATT_STAGES + 2 + 3;
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

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap mq0,
                        const __grid_constant__ CUtensorMap mq1,
                        const __grid_constant__ CUtensorMap mk0,
                        const __grid_constant__ CUtensorMap mk1,
                        const __grid_constant__ CUtensorMap mv0,
                        const __grid_constant__ CUtensorMap mv1, const AttnParams p) {
  using L = AttnSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ATT_STAGES;
  uint64_t* s_full = kv_empty + ATT_STAGES;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int qseg = (static_cast<int>(blockIdx.x) < p.q_tiles[0]) ? 0 : 1;
  const int qtile = static_cast<int>(blockIdx.x) - (qseg ? p.q_tiles[0] : 0);
  const int nblk = p.kv_blocks[0] + (p.nkv_seg > 1 ? p.kv_blocks[1] : 0);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ATT_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // tensor memory columns: S0 [0,128), S1 [128,256), O [256,384)
  const uint32_t O_COL = 256;

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap* mq = qseg ? &mq1 : &mq0;
      uint8_t* sq = smem + L::Q_OFF;
      mbar_expect_tx(q_full, 2 * L::HALF);
      tma_load_4d(sq, mq, q_full, 0, qtile * ATT_BM, head, batch);
      tma_load_4d(sq + L::HALF, mq, q_full, 64, qtile * ATT_BM, head, batch);
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int stage = j % ATT_STAGES;
        const uint32_t parity = (j / ATT_STAGES) & 1;
        if (!mbar_wait(&kv_empty[stage], parity ^ 1u, abort_flag)) break;
        const int kseg = (j < p.kv_blocks[0]) ? 0 : 1;
        const int kb = j - (kseg ? p.kv_blocks[0] : 0);
        const CUtensorMap* mk = kseg ? &mk1 : &mk0;
        const CUtensorMap* mv = kseg ? &mv1 : &mv0;
        uint8_t* sk = smem + L::KV_OFF + stage * L::STAGE;
        uint8_t* sv = sk + 2 * L::HALF;
        mbar_expect_tx(&kv_full[stage], 4 * L::HALF);
        const int t0 = kb * ATT_BN;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
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
      constexpr uint32_t idesc_o = idesc_bf16(ATT_BM, ATT_D) | (1u << 16);  // B (V) MN-major
      const uint32_t sq = smem_u32(smem + L::Q_OFF);
      const uint32_t sp = smem_u32(smem + L::P_OFF);
      bool ok = mbar_wait(q_full, 0, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int stage = j % ATT_STAGES;
        if (!mbar_wait(&kv_full[stage], (j / ATT_STAGES) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + L::KV_OFF + stage * L::STAGE);
        const uint32_t d_tmem = tmem + (j & 1) * ATT_BN;
#pragma unroll
        for (int kk = 0; kk < ATT_D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::HALF + (kk & 3) * 32;
          umma_bf16(d_tmem, sdesc_k128(sq + off), sdesc_k128(sk + off), idesc_s,
                    kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok && nblk > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk && !issue_s(j + 1)) break;
        if (!mbar_wait(p_full, j & 1, abort_flag)) break;
        tc_fence_after();
        const int stage = j % ATT_STAGES;
        const uint32_t sv = smem_u32(smem + L::KV_OFF + stage * L::STAGE + 2 * L::HALF);
#pragma unroll
        for (int kk = 0; kk < ATT_BN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * L::HALF + (kk & 3) * 32;
          umma_bf16(tmem + O_COL, sdesc_k128(sp + poff), sdesc_mn128(sv + kk * 2048, L::HALF),
                    idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[stage]);
        umma_commit(o_done);
      }
      umma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 200000000ull) {
      }
    }
  } else {
    // softmax warps 2..5: one query row per thread
    const int quarter = warp & 3;
    const int row = quarter * 32 + static_cast<int>(lane);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;  // running max of s * scale * log2(e)
    float l_run = 0.0f;
    uint8_t* sp = smem + L::P_OFF;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kseg = (j < p.kv_blocks[0]) ? 0 : 1;
      const int kb = j - (kseg ? p.kv_blocks[0] : 0);
      const int valid = min(ATT_BN, p.kv_tokens[kseg] - kb * ATT_BN);
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + (j & 1) * ATT_BN + c * 32, sr[c]);
      tmem_wait_ld();
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = __uint_as_float(sr[c][i]);
          if (c * 32 + i >= valid) v = -INFINITY;
          sr[c][i] = __float_as_uint(v);
          mx = fmaxf(mx, v);
        }
      }
      const float m_blk = mx * sl2;
      if (j > 0) {
        if (!mbar_wait(o_done, (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool need = m_blk > m_run + 8.0f;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2_approx(m_run - m_blk) : 1.0f;
          if (need) {
            m_run = m_blk;
            l_run *= alpha;
          }
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_base + O_COL + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tmem + lane_base + O_COL + c * 32, o);
          }
          tmem_wait_st();
        }
      } else {
        m_run = m_blk;
      }
      // P = exp2(s * scale * log2 e - m_run), rounded to bf16 for the MMA; l sums the same
      // rounded values.
      float lsum = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float s0 = __uint_as_float(sr[c][2 * i]);
          const float s1 = __uint_as_float(sr[c][2 * i + 1]);
          const float p0 = ex2_approx(fmaf(s0, sl2, -m_run));
          const float p1 = ex2_approx(fmaf(s1, sl2, -m_run));
          packed[i] = pack_bf16x2(p0, p1);
          const float2 r = unpack_bf16x2(packed[i]);
          lsum += r.x + r.y;
        }
        // keys c*32 .. c*32+31 live in half (c >> 1), 16-byte chunks (c & 1) * 4 .. + 3
        uint8_t* rowp = sp + (c >> 1) * L::HALF + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c & 1) * 4 + q) ^ (row & 7);
          *reinterpret_cast<uint4*>(rowp + chunk * 16) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      l_run += lsum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nblk > 0 && mbar_wait(o_done, (nblk - 1) & 1, abort_flag)) {
      tc_fence_after();
      const int t = qtile * ATT_BM + row;
      const bool store = t < p.q_tokens[qseg];
      const float inv_l = 1.0f / l_run;
      // Optional head gate: bf16(bf16(O / l) * gate[t, head])
      // (kinomlx/models/ltx2/transformer/attention.py:364-368).
      const __nv_bfloat16* gp = p.gate[qseg];
      const float gv = (gp != nullptr && store)
                           ? __bfloat162float(gp[static_cast<int64_t>(batch) * p.bs_gate[qseg] +
                                                 static_cast<int64_t>(t) * p.ld_gate[qseg] + head])
                           : 1.0f;
      auto fin = [&](uint32_t raw) -> float {
        const float o = __uint_as_float(raw) * inv_l;
        return gp != nullptr ? bf16_round(bf16_round(o) * gv) : o;
      };
      __nv_bfloat16* dst = p.out[qseg] + static_cast<int64_t>(batch) * p.bs_out[qseg] +
                           static_cast<int64_t>(t) * p.ld_out[qseg] + head * ATT_D;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + O_COL + c * 32, o);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 w;
            w.x = pack_bf16x2(fin(o[g * 8 + 0]), fin(o[g * 8 + 1]));
            w.y = pack_bf16x2(fin(o[g * 8 + 2]), fin(o[g * 8 + 3]));
            w.z = pack_bf16x2(fin(o[g * 8 + 4]), fin(o[g * 8 + 5]));
            w.w = pack_bf16x2(fin(o[g * 8 + 6]), fin(o[g * 8 + 7]));
            *reinterpret_cast<uint4*>(dst + c * 32 + g * 8) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace kino
