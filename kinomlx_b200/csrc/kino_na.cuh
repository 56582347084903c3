// Exact 3-D neighborhood attention on tcgen05 for 64-wide heads, fp16 in and out: the device form
// of kinomlx/models/ltx2/kernels/neighborhood_attention.py (the LTX-2.5 diffusion video decoder's
// attention). Every query of a (T, H, W) token grid attends to the KT x KH x KW keys of its
// window, which keeps its full size at the grid edges by shifting inward: on an axis of length L
// the window of position i starts at clamp(i - K / 2, 0, L - K). Operands are token-major
// (batch, T, H, W, heads, 64), the queries already scaled (the decoder scales them by 64^-1/2);
// scores and softmax in fp32 (exp2 domain), P stored as fp16 for the PV product, the output
// rounded to fp16 once.
//
// One work item = (batch, head, query box of 4 x 4 x 16 = 256 tokens) = two 128-query tiles,
// frames t0, t0 + 1 (A) and t0 + 2, t0 + 3 (B). The item's keys are the union of its queries'
// windows, an axis-aligned box inside the grid; it is walked in stages of 1 x 4 x 32 = 128 keys
// (a 5-D TMA box: head dim, head, W, H, batch * T) through a two-slot ring, and every stage
// feeds both tiles (the dense kernel's ping-pong: the MMA warp computes one tile's products while
// the softmax warps work on the other's), so each loaded key serves 256 queries. Each stage is
// masked per (query, key) by the query's window: a frame test and two row tests per query and
// stage and a 32-bit mask of the window's columns. One persistent CTA per SM walks the items;
// Q tiles are double-buffered so the next item's Q loads and first products overlap the
// current epilogue.
#pragma once
#include "kino_sol.cuh"

namespace kino {

constexpr int NA_QT = 4, NA_QH = 4, NA_QW = 16;  // query box (256 tokens = tiles A and B)
constexpr int NA_TILE_T = 2;                      // frames per 128-query tile
constexpr int NA_KH = 4, NA_KW = 32;             // key stage box (one frame, 128 tokens)

struct NaParams {
  int batch, frames, height, width, heads;
  int kt, kh, kw;                // window
  int boxes_t, boxes_h, boxes_w;  // query boxes per axis
  float scale_log2;               // log2(e): the queries arrive scaled
  __half* out;                    // fp16, or bf16 bits when out_bf16
  int out_bf16;
};

// Shared memory: Q tiles [buffer][tile] (16 KB each), the K/V ring [slot] (16 + 16 KB), the
// softmax exchange areas, barriers; padded past half an SM's shared memory, so that a second
// CTA never lands on an SM whose tensor memory the first one holds for its whole run.
struct NaSmem {
  static constexpr int TILE = 128 * 64 * 2;  // 128 rows x 64 fp16 = 16 KB
  static constexpr int Q_OFF = 0;            // buffer b, tile t at Q_OFF + (2 b + t) TILE
  static constexpr int KV_OFF = 4 * TILE;    // slot s: K at KV_OFF + 2 s TILE, V after it
  static constexpr int X_OFF = KV_OFF + 4 * TILE;
  static constexpr int L_OFF = X_OFF + 2 * 2 * 2 * 128 * 4;
  static constexpr int BAR_OFF = L_OFF + 2 * 2 * 128 * 4;
  // q_full[2], q_empty[2], kv_full[2], kv_empty[2], s_full[2], p_full[2], o_done, drain,
  // xbar[4][2][2], lbar[4]
  static constexpr int NBAR = 12 + 2 + 16 + 4;
  static constexpr int USED = BAR_OFF + NBAR * 8 + 16 + 1024;
  static constexpr int TOTAL = USED > 120 * 1024 ? USED : 120 * 1024;
};

// The item's key union on one axis: [first window start, last window end) of query positions
// [q0, q1) clipped to the axis.
__device__ __forceinline__ int2 na_union(int q0, int q1, int length, int k) {
  const int a = min(max(q0 - k / 2, 0), length - k);
  const int last = min(q1, length) - 1;
  const int b = min(max(last - k / 2, 0), length - k) + k;
  return make_int2(a, b);
}

__device__ __forceinline__ int na_start(int i, int length, int k) {
  return min(max(i - k / 2, 0), length - k);
}

struct NaItem {
  int b, head, t0, h0, w0;  // query box origin
  int2 ut, uh, uw;          // key union
  int nh, nw, stages;       // stage boxes per row / column, stages in all
};

__device__ __forceinline__ NaItem na_item(const NaParams& p, int it) {
  NaItem m;
  const int per_head = p.boxes_t * p.boxes_h * p.boxes_w;
  const int bh = it / per_head, box = it % per_head;
  m.b = bh / p.heads;
  m.head = bh % p.heads;
  m.t0 = (box / (p.boxes_h * p.boxes_w)) * NA_QT;
  m.h0 = ((box / p.boxes_w) % p.boxes_h) * NA_QH;
  m.w0 = (box % p.boxes_w) * NA_QW;
  m.ut = na_union(m.t0, m.t0 + NA_QT, p.frames, p.kt);
  m.uh = na_union(m.h0, m.h0 + NA_QH, p.height, p.kh);
  m.uw = na_union(m.w0, m.w0 + NA_QW, p.width, p.kw);
  m.nh = (m.uh.y - m.uh.x + NA_KH - 1) / NA_KH;
  m.nw = (m.uw.y - m.uw.x + NA_KW - 1) / NA_KW;
  m.stages = (m.ut.y - m.ut.x) * m.nh * m.nw;
  return m;
}

// stage s of an item: the key box origin (frame, row, column)
__device__ __forceinline__ int3 na_stage(const NaItem& m, int s) {
  const int per_t = m.nh * m.nw;
  return make_int3(m.ut.x + s / per_t, m.uh.x + ((s / m.nw) % m.nh) * NA_KH,
                   m.uw.x + (s % m.nw) * NA_KW);
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    na_attention_kernel(const __grid_constant__ CUtensorMap mq,
                        const __grid_constant__ CUtensorMap mk,
                        const __grid_constant__ CUtensorMap mv, const NaParams p) {
  using L = NaSmem;
  constexpr int D = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;        // [buffer]
  uint64_t* q_empty = bars + 2;   // [buffer]
  uint64_t* kv_full = bars + 4;   // [slot]
  uint64_t* kv_empty = bars + 6;  // [slot]
  uint64_t* s_full = bars + 8;    // [tile]
  uint64_t* p_full = bars + 10;   // [tile]
  uint64_t* o_done = bars + 12;
  uint64_t* drain = bars + 13;
  uint64_t* xbar = bars + 14;     // [quarter][tile][parity]
  uint64_t* lbar = xbar + 16;     // [quarter]
  float* xmax = reinterpret_cast<float*>(smem + L::X_OFF);
  float* xsum = reinterpret_cast<float*>(smem + L::L_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  const int items = p.batch * p.heads * p.boxes_t * p.boxes_h * p.boxes_w;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 16; ++i) mbar_init(&xbar[i], 64);
    for (int i = 0; i < 4; ++i) mbar_init(&lbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&mq);
    tma_prefetch(&mk);
    tma_prefetch(&mv);
  }
  griddep_wait();
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
      int g = 0;  // stages issued over all items: ring slot g % 2, phase (g / 2) % 2
      int j = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++j) {
        const NaItem m = na_item(p, it);
        const int buf = j & 1;
        const uint32_t use = static_cast<uint32_t>(j >> 1) & 1u;
        if (!mbar_wait(&q_empty[buf], use ^ 1u, abort_flag)) break;
        const int bt = m.b * p.frames;
        mbar_expect_tx(&q_full[buf], 2 * L::TILE);
        for (int t = 0; t < 2; ++t)
          tma_load_5d(smem + L::Q_OFF + (2 * buf + t) * L::TILE, &mq, &q_full[buf], 0, m.head,
                      m.w0, m.h0, bt + m.t0 + t * NA_TILE_T);
        for (int s = 0; s < m.stages; ++s, ++g) {
          const int slot = g & 1;
          if (!mbar_wait(&kv_empty[slot], (static_cast<uint32_t>(g >> 1) & 1u) ^ 1u, abort_flag))
            break;
          const int3 o = na_stage(m, s);
          uint8_t* sk = smem + L::KV_OFF + slot * 2 * L::TILE;
          mbar_expect_tx(&kv_full[slot], 2 * L::TILE);
          tma_load_5d(sk, &mk, &kv_full[slot], 0, m.head, o.z, o.y, bt + o.x);
          tma_load_5d(sk + L::TILE, &mv, &kv_full[slot], 0, m.head, o.z, o.y, bt + o.x);
        }
      }
      if (*abort_flag) {
        // after a timeout, give copies still in flight a bounded moment to land
        const uint64_t t0 = global_ns();
        while (global_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(ATT_BM, ATT_BN);
      constexpr uint32_t idesc_o = idesc_f16(ATT_BM, D) | (1u << 16);  // B (V) MN-major
      int g = 0;   // stages consumed over all items (ring slot and phase)
      int pc = 0;  // P signals consumed per tile (both tiles advance together)
      bool ok = true;
      int j = 0;
      for (int it = blockIdx.x; ok && it < items; it += gridDim.x, ++j) {
        const NaItem m = na_item(p, it);
        const int buf = j & 1;
        const uint32_t use = static_cast<uint32_t>(j >> 1) & 1u;
        if (!mbar_wait(&q_full[buf], use, abort_flag)) break;
        const int nst = m.stages;
        auto s_mma = [&](int t, int slot) {  // S_t = Q_t K^T of the stage in `slot`
          const uint32_t sq = smem_u32(smem + L::Q_OFF + (2 * buf + t) * L::TILE);
          const uint32_t sk = smem_u32(smem + L::KV_OFF + slot * 2 * L::TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_bf16(tmem + t * 128, sdesc_k128(sq + kk * 32), sdesc_k128(sk + kk * 32), idesc_s,
                      kk > 0 ? 1u : 0u);
          umma_commit(&s_full[t]);
        };
        auto pv_mma = [&](int t, int slot, bool first) {  // O_t += P_t V of the stage in `slot`
          const uint32_t sv = smem_u32(smem + L::KV_OFF + slot * 2 * L::TILE + L::TILE);
#pragma unroll
          for (int kk = 0; kk < ATT_BN / 16; ++kk)
            umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8 + (kk >= 4 ? 32 : 0),
                         sdesc_mn128(sv + kk * 2048, L::TILE), idesc_o,
                         (!first || kk > 0) ? 1u : 0u);
        };
        auto wait_kv = [&](int gg) {
          const bool got = mbar_wait(&kv_full[gg & 1], static_cast<uint32_t>(gg >> 1) & 1u,
                                     abort_flag);
          if (got) tc_fence_after();
          return got;
        };
        ok = wait_kv(g);
        if (ok) {
          s_mma(0, g & 1);
          s_mma(1, g & 1);
        }
        for (int s = 0; ok && s < nst; ++s) {
          const int slot = (g + s) & 1;
          const bool more = s + 1 < nst;
          for (int t = 0; t < 2 && ok; ++t) {
            if (!mbar_wait(&p_full[t], static_cast<uint32_t>(pc) & 1u, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            pv_mma(t, slot, s == 0);
            if (t == 1) umma_commit(&kv_empty[slot]);
            if (more) {
              if (t == 0) {
                ok = wait_kv(g + s + 1);
                if (!ok) break;
              }
              s_mma(t, (g + s + 1) & 1);
            }
          }
          ++pc;
        }
        if (!ok) break;
        g += nst;
        umma_commit(&q_empty[buf]);
        umma_commit(o_done);
      }
      umma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 200000000ull) {
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + static_cast<int>(lane);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    int pc = 0;  // stages seen over all items (barrier and buffer phases)
    bool ok = true;
    int j = 0;
    for (int it = blockIdx.x; ok && it < items; it += gridDim.x, ++j) {
      const NaItem m = na_item(p, it);
      // this row's query in each tile and the starts of its windows
      int qt[2], st[2];
      const int qh = m.h0 + (row / NA_QW) % NA_QH;
      const int qw = m.w0 + row % NA_QW;
      const int sh = na_start(qh, p.height, p.kh);
      const int sw = na_start(qw, p.width, p.kw);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        qt[t] = m.t0 + t * NA_TILE_T + row / (NA_QH * NA_QW);
        st[t] = na_start(qt[t], p.frames, p.kt);
      }
      const int nst = m.stages;
      float m_run[2] = {-INFINITY, -INFINITY};
      float l_run[2] = {0.0f, 0.0f};
      for (int s = 0; s < nst && ok; ++s, ++pc) {
        const int3 o = na_stage(m, s);
        // this warp's 64 keys: rows o.y + 2 half + c, columns o.z + i
        bool hok[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int kr = o.y + 2 * half + c;
          hok[c] = kr >= sh && kr < sh + p.kh;
        }
        const int lo = min(max(sw - o.z, 0), 32), hi = min(max(sw + p.kw - o.z, 0), 32);
        const uint32_t below_hi = hi >= 32 ? 0xFFFFFFFFu : ((1u << hi) - 1u);
        const uint32_t below_lo = lo >= 32 ? 0xFFFFFFFFu : ((1u << lo) - 1u);
        const uint32_t wmask = below_hi & ~below_lo;
        for (int t = 0; t < 2 && ok; ++t) {
          const bool tok = o.x >= st[t] && o.x < st[t] + p.kt;
          if (!mbar_wait(&s_full[t], static_cast<uint32_t>(pc) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t s_col = tmem + lane_base + t * 128 + half * 64;
          uint32_t sr[2][32];
          tmem_ld32(s_col, sr[0]);
          tmem_ld32(s_col + 32, sr[1]);
          tmem_wait_ld();
          const uint32_t keep0 = (tok && hok[0]) ? wmask : 0u;
          const uint32_t keep1 = (tok && hok[1]) ? wmask : 0u;
          // a warp whose 32 rows see none of its 64 keys skips the max and the exponentials
          // (its P is 0), but still exchanges its maximum and rescales with its partner warp
          const bool live = __any_sync(0xffffffffu, (keep0 | keep1) != 0u);
          float mine = -INFINITY;
          if (live) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const uint32_t keep = c ? keep1 : keep0;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (!((keep >> i) & 1u)) sr[c][i] = __float_as_uint(-INFINITY);
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
            mine = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
          }
          float* xm = xmax + (t * 2 + (pc & 1)) * 256;
          xm[half * 128 + row] = mine;
          uint64_t* xb = &xbar[(quarter * 2 + t) * 2 + (pc & 1)];
          mbar_arrive(xb);
          if (!mbar_wait(xb, static_cast<uint32_t>(pc >> 1) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          const float m_blk = fmaxf(mine, xm[(1 - half) * 128 + row]);
          float alpha = 1.0f;
          bool rescale = false;
          if (s > 0) {
            const bool need = m_blk > m_run[t] + 8.0f;
            rescale = __any_sync(0xffffffffu, need);
            if (need) {
              alpha = ex2_approx(m_run[t] - m_blk);  // 0 while the row had no key yet
              m_run[t] = m_blk;
              l_run[t] *= alpha;
            }
          } else {
            m_run[t] = m_blk;
          }
          // a row with no key so far subtracts 0: its exponentials are all 0 (or 2^-126)
          const float msub = m_run[t] == -INFINITY ? 0.0f : m_run[t];
          const uint64_t sc2 = f2_pack(sl2, sl2);
          const uint64_t negm = f2_pack(-msub, -msub);
          if (live) {
            uint64_t lsum2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
              uint32_t packed[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int jj = q8 * 8 + u;
                const uint32_t* v = sr[jj >> 4];
                const int e = (2 * jj) & 31;
                const uint64_t xs =
                    f2_fma(f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sc2, negm);
                uint64_t ev;
                if ((ATT_EMU_MASK >> (jj & 7)) & 1) {
                  ev = exp2_poly_x2(xs);
                } else {
                  const float2 xv = f2_unpack(xs);
                  ev = f2_pack(ex2_approx(xv.x), ex2_approx(xv.y));
                }
                lsum2[u & 1] = f2_add(lsum2[u & 1], ev);
                const float2 e2 = f2_unpack(ev);
                packed[u] = pack_f16x2(e2.x, e2.y);
              }
              tmem_st8(s_col + q8 * 8, packed);
            }
            const float2 ls = f2_unpack(f2_add(lsum2[0], lsum2[1]));
            l_run[t] += ls.x + ls.y;
          } else {
            const uint32_t zeros[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) tmem_st8(s_col + q8 * 8, zeros);
          }
          if (rescale) {
            const uint32_t o_col = tmem + lane_base + 256 + t * 128 + half * (D / 2);
            uint32_t ov[32];
            tmem_ld32(o_col, ov);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              ov[jj] = __float_as_uint(__uint_as_float(ov[jj]) * alpha);
            tmem_st32(o_col, ov);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[t]);
        }
      }
      if (!ok) break;
      for (int t = 0; t < 2; ++t) xsum[(t * 2 + half) * 128 + row] = l_run[t];
      mbar_arrive(&lbar[quarter]);
      if (!mbar_wait(&lbar[quarter], static_cast<uint32_t>(j) & 1u, abort_flag) ||
          !mbar_wait(o_done, static_cast<uint32_t>(j) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int t = 0; t < 2; ++t) {
        const float inv_l = 1.0f / (l_run[t] + xsum[(t * 2 + 1 - half) * 128 + row]);
        uint32_t ov[32];
        tmem_ld32(tmem + lane_base + 256 + t * 128 + half * (D / 2), ov);
        tmem_wait_ld();
        if (qt[t] < p.frames && qh < p.height && qw < p.width) {
          const int64_t tok = ((static_cast<int64_t>(m.b) * p.frames + qt[t]) * p.height + qh) *
                                  p.width + qw;
          __half* dst = p.out + (tok * p.heads + m.head) * D + half * (D / 2);
          uint32_t w16[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float o0 = __uint_as_float(ov[2 * e]) * inv_l;
            const float o1 = __uint_as_float(ov[2 * e + 1]) * inv_l;
            w16[e] = p.out_bf16 ? pack_bf16x2(o0, o1) : pack_f16x2(o0, o1);
          }
          store_row32(reinterpret_cast<__nv_bfloat16*>(dst), w16, 32);
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
