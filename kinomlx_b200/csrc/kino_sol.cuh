// Sol-Attn routed block-sparse attention for 128-wide heads on tcgen05: the device form of
// kinomlx/models/ltx2/kernels/sol_attention.py:98-272 (the published Sol-Attn of NVlabs' Sana
// Sol-Engine): tokens in 64-token blocks along a given routing order (normally a 3-D Morton
// curve); each query block scores every key block by its mean query against the block's mean
// key and routes the blocks above mean + tau * std of those scores (diagonal key covariance),
// plus itself and both neighbours; routed blocks are attended exactly, every other block through
// its mean key (score + log2 of the block's length) and mean value, all in one softmax.
//
// Three launches:
//   sol_prepare_kernel   gather q, k, v into routing order as fp16 (saturating at 65504, as the
//                        reference's kernel converts them), and the 64-token block means: fp32
//                        query means, key / value means rounded to the input dtype, then fp16
//   sol_route_kernel     per (head, query block): the routing row as 32-bit mask words
//   sol_union_kernel     per (head, CTA): the ascending list of key blocks routed by any of the
//                        CTA's four query blocks
//   sol_attention_kernel the attention: attention_tc_kernel's pipeline (two 128-query tiles =
//                        four Sol blocks per CTA in ping-pong, TMA / MMA / eight softmax warps,
//                        S and O in tensor memory, P back over S) on fp16 operands, with the K/V
//                        producer walking the CTA's block list (two 64-key blocks per 128-key
//                        stage) and then the centroid keys (every key block's mean, 128 per
//                        stage). Each softmax warp covers one 64-key block per stage, so routing
//                        is one mask bit per (row, stage half) for exact blocks and one per
//                        (row, key) for centroids (a row's routed blocks are excluded there).
//                        Output rows go back to their input positions, in the input dtype, with
//                        the optional per-head gate.
#pragma once
#include <cuda_fp16.h>

#include "kino_attention.cuh"

namespace kino {

constexpr int SOL_BLOCK = 64;
constexpr int SOL_MAX_WORDS = 16;  // mask words per query block: at most 512 blocks
constexpr int SOL_QBLOCKS = 4;     // query blocks per attention CTA (two 128-row tiles)

__device__ __forceinline__ float sol_sat(float x) { return fminf(fmaxf(x, -65504.0f), 65504.0f); }

template <typename In>
__device__ __forceinline__ float sol_round_in(float x) {
  if constexpr (sizeof(In) == 2 && std::is_same<In, __half>::value)
    return __half2float(__float2half_rn(x));
  else
    return __bfloat162float(__float2bfloat16_rn(x));
}

template <typename In>
__device__ __forceinline__ void sol_load8(const In* p, float (&f)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<In, __half>::value) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    } else {
      const float2 v = unpack_bf16x2(w[i]);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// grid (blocks, heads), 128 threads: 16 threads per token row (8 columns each), 8 rows per pass.
template <typename In>
__global__ void __launch_bounds__(128)
    sol_prepare_kernel(const In* __restrict__ q, const In* __restrict__ k,
                       const In* __restrict__ v, int64_t ldq, int64_t ldk, int64_t ldv,
                       const int* __restrict__ order, int tokens, int heads,
                       __half* __restrict__ q16, __half* __restrict__ k16,
                       __half* __restrict__ v16, float* __restrict__ qmean,
                       __half* __restrict__ kmean, __half* __restrict__ vmean) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[3][8][128];
  const int b = blockIdx.x, h = blockIdx.y, nb = gridDim.x;
  const int cv = threadIdx.x & 15, rg = threadIdx.x >> 4;
  const int n = min(SOL_BLOCK, tokens - b * SOL_BLOCK);
  const int64_t width = static_cast<int64_t>(heads) * 128;
  const int col = h * 128 + cv * 8;
  float acc[3][8];
#pragma unroll
  for (int s = 0; s < 3; ++s)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[s][j] = 0.0f;
  for (int i = rg; i < n; i += 8) {
    const int dst = b * SOL_BLOCK + i;
    const int64_t src = order[dst];
    if (src < 0 || src >= tokens) {  // not a permutation of the rows: report, never read past
      atomicExch(&g_device_error, 1);
      continue;
    }
    const In* srcs[3] = {q + src * ldq + col, k + src * ldk + col, v + src * ldv + col};
    __half* dsts[3] = {q16 + dst * width + col, k16 + dst * width + col, v16 + dst * width + col};
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      float f[8];
      sol_load8(srcs[s], f);
      uint4 w;
      w.x = pack_f16x2(sol_sat(f[0]), sol_sat(f[1]));
      w.y = pack_f16x2(sol_sat(f[2]), sol_sat(f[3]));
      w.z = pack_f16x2(sol_sat(f[4]), sol_sat(f[5]));
      w.w = pack_f16x2(sol_sat(f[6]), sol_sat(f[7]));
      *reinterpret_cast<uint4*>(dsts[s]) = w;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[s][j] += f[j];
    }
  }
#pragma unroll
  for (int s = 0; s < 3; ++s)
#pragma unroll
    for (int j = 0; j < 8; ++j) red[s][rg][cv * 8 + j] = acc[s][j];
  __syncthreads();
  const int c = threadIdx.x;
  float sum[3];
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    float t = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) t += red[s][r][c];
    sum[s] = t / static_cast<float>(n);
  }
  const int64_t m = (static_cast<int64_t>(h) * nb + b) * 128 + c;
  qmean[m] = sum[0];
  kmean[m] = __float2half_rn(sol_sat(sol_round_in<In>(sum[1])));
  vmean[m] = __float2half_rn(sol_sat(sol_round_in<In>(sum[2])));
}

// grid (ceil(blocks / 8), heads), 256 threads: the routing rows of eight query blocks, one per
// warp. The key-mean center and per-dimension variance over the blocks come first (thread d < 128
// for dimension d); then each warp forms its row's limit, the row's mean score plus tau standard
// deviations under a diagonal key covariance, and scores 32 key blocks at a time (lane l takes
// block 32 i + l: a 128-long dot product against its mean key), a ballot turning the comparisons
// into mask word i (kinomlx/models/ltx2/kernels/sol_attention.py:181-216).
constexpr int SOL_ROUTE_ROWS = 8;

__global__ void __launch_bounds__(256)
    sol_route_kernel(const float* __restrict__ qmean, const __half* __restrict__ kmean, int nb,
                     int words, float log2_scale, float log2_scale_sq, float tau,
                     uint32_t* __restrict__ bits) {
  griddep_wait();
  griddep_launch();
  __shared__ float center[128], var[128];
  __shared__ float qs[SOL_ROUTE_ROWS][128];
  const int h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __half* kh = kmean + static_cast<int64_t>(h) * nb * 128;
  if (tid < 128) {
    float s = 0.0f;
    for (int b = 0; b < nb; ++b) s += __half2float(kh[b * 128 + tid]);
    const float c = s / static_cast<float>(nb);
    float s2 = 0.0f;
    for (int b = 0; b < nb; ++b) {
      const float dl = __half2float(kh[b * 128 + tid]) - c;
      s2 += dl * dl;
    }
    center[tid] = c;
    var[tid] = s2 / static_cast<float>(nb);
  }
  const int a0 = blockIdx.x * SOL_ROUTE_ROWS;
  for (int i = tid; i < SOL_ROUTE_ROWS * 128; i += 256) {
    const int r = i >> 7, a = a0 + r;
    qs[r][i & 127] = a < nb ? qmean[(static_cast<int64_t>(h) * nb + a) * 128 + (i & 127)] : 0.0f;
  }
  __syncthreads();
  const int a = a0 + warp;
  if (a >= nb) return;
  const float* q = qs[warp];
  float rm = 0.0f, rv = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    rm += q[d] * center[d];
    rv += q[d] * q[d] * var[d];
  }
  const float raw_mean = warp_sum_f(rm);
  const float raw_var = warp_sum_f(rv);
  const float variance = fmaxf(raw_var, 0.0f) * log2_scale_sq;
  const float limit = raw_mean * log2_scale + tau * sqrtf(variance + 1.0e-6f);
  uint32_t* row = bits + (static_cast<int64_t>(h) * nb + a) * words;
  for (int w = 0; w < words; ++w) {
    const int b = w * 32 + lane;
    bool routed = false;
    if (b < nb) {
      const uint4* kr = reinterpret_cast<const uint4*>(kh + b * 128);
      float dot = 0.0f;
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        const uint4 raw = kr[c];
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kv = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
          dot = fmaf(q[c * 8 + 2 * e], kv.x, dot);
          dot = fmaf(q[c * 8 + 2 * e + 1], kv.y, dot);
        }
      }
      routed = (b >= a - 1 && b <= a + 1) || dot * log2_scale > limit;
    }
    const uint32_t word = __ballot_sync(0xffffffffu, routed);
    if (lane == 0) row[w] = word;
  }
}

// grid (CTAs per head, heads), 32 threads: the union of the routing rows of query blocks
// 4c .. 4c + 3 as an ascending block list and its length.
__global__ void __launch_bounds__(32)
    sol_union_kernel(const uint32_t* __restrict__ bits, int nb, int words,
                     int* __restrict__ lists, int* __restrict__ counts) {
  griddep_wait();
  griddep_launch();
  const int c = blockIdx.x, h = blockIdx.y, ncta = gridDim.x;
  const int lane = threadIdx.x;
  uint32_t u = 0;
  if (lane < words) {
    for (int a = c * SOL_QBLOCKS; a < min(nb, (c + 1) * SOL_QBLOCKS); ++a)
      u |= bits[(static_cast<int64_t>(h) * nb + a) * words + lane];
  }
  const int n = __popc(u);
  int incl = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int at = incl - n;
  int* list = lists + (static_cast<int64_t>(h) * ncta + c) * nb;
  while (u) {
    const int bit = __ffs(u) - 1;
    u &= u - 1;
    list[at++] = lane * 32 + bit;
  }
  if (lane == 31) counts[h * ncta + c] = incl;
}

__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4)                                  // D format: f32; A, B format: f16 (0)
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

struct SolParams {
  int tokens, heads, nb, words, ncta;
  float scale_log2;  // 128^-1/2 * log2(e)
  float last_log2;   // log2 of the last block's length
  const uint32_t* bits;
  const int* lists;
  const int* counts;
  const int* order;
  void* out;
  int64_t ld_out;
  int out_f16;       // output dtype: 1 fp16, 0 bf16 (the inputs' dtype)
  const void* gate;  // optional (tokens, heads) gate in input order, input dtype
  int64_t ld_gate;
};

__global__ void __launch_bounds__(ATT_THREADS, 1)
    sol_attention_kernel(const __grid_constant__ CUtensorMap mq,
                         const __grid_constant__ CUtensorMap mk,
                         const __grid_constant__ CUtensorMap mv,
                         const __grid_constant__ CUtensorMap mkc,
                         const __grid_constant__ CUtensorMap mvc, const SolParams p) {
  using L = AttnSmem;
  constexpr int D = 128;
  constexpr int NH = 2;
  constexpr int SUB = 64 * 128;  // one 64-row box of a 64-wide swizzled half: 8 KB
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ATT_STAGES;
  uint64_t* s_full = kv_empty + ATT_STAGES;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 1;
  uint64_t* xbar = drain + 1;
  uint64_t* lbar = xbar + 16;
  float* xmax = reinterpret_cast<float*>(smem + L::X_OFF);
  float* xsum = reinterpret_cast<float*>(smem + L::L_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // routing words of the CTA's four query blocks and its block list, after the barrier block
  uint32_t* rwords = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBAR * 8 + 16);
  int* slist = reinterpret_cast<int*>(rwords + SOL_QBLOCKS * SOL_MAX_WORDS);

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  const int cta = blockIdx.x;
  const int head = blockIdx.y;
  const int row0 = cta * 256;  // tile t covers routed rows [row0 + 128 t, row0 + 128 t + 128)
  const bool has_b = row0 + 128 < p.tokens;
  const int ntile = has_b ? 2 : 1;
  const int* list = p.lists + (static_cast<int64_t>(head) * p.ncta + cta) * p.nb;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ATT_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 8);
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 16; ++i) mbar_init(&xbar[i], 64);
    for (int i = 0; i < 4; ++i) mbar_init(&lbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  griddep_wait();
  if (threadIdx.x < SOL_QBLOCKS * SOL_MAX_WORDS) {
    const int qb = cta * SOL_QBLOCKS + threadIdx.x / SOL_MAX_WORDS;
    const int w = threadIdx.x % SOL_MAX_WORDS;
    rwords[threadIdx.x] = (qb < p.nb && w < p.words)
                              ? p.bits[(static_cast<int64_t>(head) * p.nb + qb) * p.words + w]
                              : 0u;
  }
  const int count = p.counts[head * p.ncta + cta];
  for (int i = threadIdx.x; i < count; i += blockDim.x) slist[i] = list[i];
  const int ns = (count + 1) / 2;               // exact stages: two 64-key blocks each
  const int nblk = ns + (p.nb + 127) / 128;     // then the centroid stages
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
      mbar_expect_tx(q_full, ntile * NH * L::HALF);
      for (int t = 0; t < ntile; ++t) {
        uint8_t* sq = smem + L::Q_OFF + t * 2 * L::HALF;
        tma_load_4d(sq, &mq, q_full, 0, row0 + t * 128, head, 0);
        tma_load_4d(sq + L::HALF, &mq, q_full, 64, row0 + t * 128, head, 0);
      }
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int stage = j % ATT_STAGES;
        const uint32_t parity = (j / ATT_STAGES) & 1;
        if (!mbar_wait(&kv_empty[stage], parity ^ 1u, abort_flag)) break;
        uint8_t* sk = smem + L::KV_OFF + stage * L::STAGE;
        uint8_t* sv = sk + 2 * L::HALF;
        mbar_expect_tx(&kv_full[stage], 2 * NH * L::HALF);
        if (j < ns) {
          const int kb0 = slist[2 * j];
          const int kb1 = 2 * j + 1 < count ? slist[2 * j + 1] : kb0;  // a masked stand-in
#pragma unroll
          for (int h2 = 0; h2 < NH; ++h2) {
            tma_load_4d(sk + h2 * L::HALF, &mk, &kv_full[stage], h2 * 64, kb0 * 64, head, 0);
            tma_load_4d(sk + h2 * L::HALF + SUB, &mk, &kv_full[stage], h2 * 64, kb1 * 64, head, 0);
            tma_load_4d(sv + h2 * L::HALF, &mv, &kv_full[stage], h2 * 64, kb0 * 64, head, 0);
            tma_load_4d(sv + h2 * L::HALF + SUB, &mv, &kv_full[stage], h2 * 64, kb1 * 64, head, 0);
          }
        } else {
          const int c0 = (j - ns) * 128;
#pragma unroll
          for (int h2 = 0; h2 < NH; ++h2) {
            tma_load_3d(sk + h2 * L::HALF, &mkc, &kv_full[stage], h2 * 64, c0, head);
            tma_load_3d(sk + h2 * L::HALF + SUB, &mkc, &kv_full[stage], h2 * 64, c0 + 64, head);
            tma_load_3d(sv + h2 * L::HALF, &mvc, &kv_full[stage], h2 * 64, c0, head);
            tma_load_3d(sv + h2 * L::HALF + SUB, &mvc, &kv_full[stage], h2 * 64, c0 + 64, head);
          }
        }
        ++issued;
      }
      if (*abort_flag) {
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
      constexpr uint32_t idesc_s = idesc_f16(ATT_BM, ATT_BN);
      constexpr uint32_t idesc_o = idesc_f16(ATT_BM, D) | (1u << 16);  // B (V) MN-major
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
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + static_cast<int>(lane);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.0f, 0.0f};
    bool ok = true;
    // one stage of this warp: 64 keys, an exact block kb (or none) or centroids c0 .. c0 + 63;
    // instantiated once per kind so that each loop's body stays compact
    auto stage = [&](const int j, auto kind) {
      constexpr bool exact = decltype(kind)::value;
      int kb = -1, nk = 0, c0 = 0;
      if constexpr (exact) {
        const int li = 2 * j + half;
        kb = li < count ? slist[li] : -1;
        nk = kb >= 0 ? min(SOL_BLOCK, p.tokens - kb * SOL_BLOCK) : 0;
      } else {
        c0 = (j - ns) * 128 + half * 64;
      }
      for (int t = 0; t < ntile; ++t) {
        if (!mbar_wait(&s_full[t], j & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t* rw = rwords + (2 * t + (row >> 6)) * SOL_MAX_WORDS;
        const uint32_t s_col = tmem + lane_base + t * 128 + half * 64;
        uint32_t sr[2][32];
        tmem_ld32(s_col, sr[0]);
        tmem_ld32(s_col + 32, sr[1]);
        tmem_wait_ld();
        // An exact block is all or nothing for a row: its logits are s * scale - m, folded into
        // one packed FMA per pair with a per-row (scale, offset) = (sl2, -m), or (0, -inf) when
        // the row does not route the block. Centroid logits carry a per-key bias (log2 of the
        // block's length) or -inf; they are formed here, already scaled.
        bool routed_row = true;
        float mine;
        if constexpr (exact) {
          routed_row = kb >= 0 && ((rw[kb >> 5] >> (kb & 31)) & 1u);
          if (nk < SOL_BLOCK) {  // the last, partial block (warp-uniform): finite sentinel
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (c * 32 + i >= nk) sr[c][i] = __float_as_uint(-1.0e30f);
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
          const float raw = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
          mine = routed_row ? raw * sl2 : -INFINITY;
        } else {
          const int w0 = c0 >> 5;
          const uint32_t words[2] = {w0 < p.words ? rw[w0] : ~0u,
                                     w0 + 1 < p.words ? rw[w0 + 1] : ~0u};
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int b = c0 + c * 32 + i;
              const float bias = b == p.nb - 1 ? p.last_log2 : 6.0f;
              const bool take = b < p.nb && !((words[c] >> i) & 1u);
              sr[c][i] = __float_as_uint(take ? fmaf(__uint_as_float(sr[c][i]), sl2, bias)
                                              : -INFINITY);
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
          mine = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        }
        float* xm = xmax + (t * 2 + (j & 1)) * 256;
        xm[half * 128 + row] = mine;
        uint64_t* xb = &xbar[(quarter * 2 + t) * 2 + (j & 1)];
        mbar_arrive(xb);
        if (!mbar_wait(xb, (j >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        const float m_blk = fmaxf(mine, xm[(1 - half) * 128 + row]);
        float alpha = 1.0f;
        bool rescale = false;
        if (j > 0) {
          const bool need = m_blk > m_run[t] + 8.0f;
          rescale = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = ex2_approx(m_run[t] - m_blk);  // 0 while the row had no logit yet
            m_run[t] = m_blk;
            l_run[t] *= alpha;
          }
        } else {
          m_run[t] = m_blk;
        }
        // a row with no logit so far subtracts 0: its exponentials are all 0 (or 2^-126)
        const float msub = m_run[t] == -INFINITY ? 0.0f : m_run[t];
        const float scl = exact ? (routed_row ? sl2 : 0.0f) : 1.0f;
        const float off = (exact && !routed_row) ? -INFINITY : -msub;
        const uint64_t sc2 = f2_pack(scl, scl);
        const uint64_t negm = f2_pack(off, off);
        uint64_t lsum2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          uint32_t packed[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int i = q8 * 8 + u;
            const uint32_t* v = sr[i >> 4];
            const int e = (2 * i) & 31;
            const uint64_t xs =
                f2_fma(f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sc2, negm);
            uint64_t ev;
            if ((ATT_EMU_MASK >> (i & 7)) & 1) {
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
    };
    for (int j = 0; j < ns && ok; ++j) stage(j, std::true_type{});
    for (int j = ns; j < nblk && ok; ++j) stage(j, std::false_type{});
    if (ok && nblk > 0) {
      for (int t = 0; t < ntile; ++t) xsum[(t * 2 + half) * 128 + row] = l_run[t];
      mbar_arrive(&lbar[quarter]);
      ok = mbar_wait(&lbar[quarter], 0, abort_flag);
    }
    if (ok && nblk > 0 && mbar_wait(o_done, 0, abort_flag)) {
      tc_fence_after();
      for (int t = 0; t < ntile; ++t) {
        const int tok = row0 + t * 128 + row;
        bool store = tok < p.tokens;
        const float inv_l = 1.0f / (l_run[t] + xsum[(t * 2 + 1 - half) * 128 + row]);
        const int64_t dst_row = store ? p.order[tok] : 0;
        if (store && (dst_row < 0 || dst_row >= p.tokens)) {
          atomicExch(&g_device_error, 1);
          store = false;
        }
        float gv = 1.0f;
        if (p.gate != nullptr && store) {
          const int64_t gi = dst_row * p.ld_gate + head;
          gv = p.out_f16 ? __half2float(static_cast<const __half*>(p.gate)[gi])
                         : __bfloat162float(static_cast<const __nv_bfloat16*>(p.gate)[gi]);
        }
        auto fin = [&](uint32_t raw) -> float {
          const float o = __uint_as_float(raw) * inv_l;
          if (p.gate == nullptr) return o;
          const float r = p.out_f16 ? __half2float(__float2half_rn(o)) : bf16_round(o);
          return r * gv;
        };
        const uint32_t o_col = tmem + lane_base + 256 + t * 128 + half * (D / 2);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
          if (store) {
            uint8_t* base = static_cast<uint8_t*>(p.out) +
                            (dst_row * p.ld_out + head * D + half * (D / 2) + c * 32) * 2;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 w;
              if (p.out_f16) {
                w.x = pack_f16x2(fin(o[g * 8 + 0]), fin(o[g * 8 + 1]));
                w.y = pack_f16x2(fin(o[g * 8 + 2]), fin(o[g * 8 + 3]));
                w.z = pack_f16x2(fin(o[g * 8 + 4]), fin(o[g * 8 + 5]));
                w.w = pack_f16x2(fin(o[g * 8 + 6]), fin(o[g * 8 + 7]));
              } else {
                w.x = pack_bf16x2(fin(o[g * 8 + 0]), fin(o[g * 8 + 1]));
                w.y = pack_bf16x2(fin(o[g * 8 + 2]), fin(o[g * 8 + 3]));
                w.z = pack_bf16x2(fin(o[g * 8 + 4]), fin(o[g * 8 + 5]));
                w.w = pack_bf16x2(fin(o[g * 8 + 6]), fin(o[g * 8 + 7]));
              }
              *reinterpret_cast<uint4*>(base + g * 16) = w;
            }
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
