// Sol-Attn routed block-sparse attention for 128-wide heads on tcgen05: the device form of
// kinomlx/models/ltx2/kernels/sol_attention.py:98-272 (the published Sol-Attn of NVlabs' Sana
// Sol-Engine): tokens in 64-token blocks along a given routing order (normally a 3-D Morton
// curve); each query block scores every key block by its mean query against the block's mean
// key and routes the blocks above mean + tau * std of those scores (diagonal key covariance),
// plus itself and both neighbours; routed blocks are attended exactly, every other block through
// its mean key (score + log2 of the block's length) and mean value, all in one softmax.
//
// Four launches:
//   sol_prepare_kernel   gather q, k, v into routing order as fp16 (saturating at 65504, as the
//                        reference's kernel converts them), and the 64-token block means: fp32
//                        query means, key / value means rounded to the input dtype, then fp16
//   sol_route_kernel     per (head, query block): the routing row as 32-bit mask words
//   sol_union_kernel     per (head, query tile): the ascending list of key blocks routed by any
//                        of the tile's two query blocks
//   sol_attention_kernel the attention: a persistent CTA per SM walks (head, query tile) items;
//                        attention_tc_kernel's roles (TMA / MMA / eight softmax warps, S and O in
//                        tensor memory, P back over S) on fp16 operands, one 128-row query tile
//                        per item whose key stages alternate between two streams (own S, O and
//                        row statistics each, merged at the end). The K/V producer walks the
//                        item's block list (two 64-key blocks per 128-key stage) and then the
//                        centroid keys (every key block's mean, 128 per stage). Each softmax warp
//                        covers one 64-key block per stage, so routing is one mask bit per (row,
//                        stage half) for exact blocks and one per (row, key) for centroids (a
//                        row's routed blocks are excluded there). Output rows go back to their
//                        input positions, in the input dtype, with the optional per-head gate.
#pragma once
#include <cuda_fp16.h>

#include "kino_attention.cuh"

namespace kino {

constexpr int SOL_BLOCK = 64;
constexpr int SOL_MAX_WORDS = 16;  // mask words per query block: at most 512 blocks
constexpr int SOL_QBLOCKS = 2;     // query blocks per attention CTA (one 128-row tile)

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

// grid (ceil(blocks / 16), heads), 256 threads: the routing rows of 16 query blocks
// (kinomlx/models/ltx2/kernels/sol_attention.py:181-216). The head's key means are staged in
// shared memory once (rows padded to 272 bytes, so a warp's 16-byte loads of 32 different rows
// meet no bank conflict), their center and per-dimension variance reduced in a fixed order, and
// each row's limit is its mean score plus tau standard deviations under a diagonal key
// covariance. Scores: a warp owns eight query rows and a 32-block word of keys, lane l key block
// 32 w + l; the eight query rows are read as broadcasts, so every lane runs 8 x 128 FMAs with no
// shuffles and a ballot per row turns the comparisons into the mask word.
constexpr int SOL_ROUTE_ROWS = 16;
constexpr int SOL_KEY_PAD = 136;  // halves per staged key-mean row

__host__ __device__ constexpr int sol_route_smem(int nb) {
  return nb * SOL_KEY_PAD * 2 + (16 * 128 + 128 + 128 + SOL_ROUTE_ROWS * 128 + SOL_ROUTE_ROWS) * 4;
}

__global__ void __launch_bounds__(256)
    sol_route_kernel(const float* __restrict__ qmean, const __half* __restrict__ kmean, int nb,
                     int words, float log2_scale, float log2_scale_sq, float tau,
                     uint32_t* __restrict__ bits) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) uint8_t rsm[];
  __half* ks = reinterpret_cast<__half*>(rsm);
  float* part = reinterpret_cast<float*>(rsm + nb * SOL_KEY_PAD * 2);
  float* center = part + 16 * 128;
  float* var = center + 128;
  float* qs = var + 128;                      // [SOL_ROUTE_ROWS][128]
  float* limit = qs + SOL_ROUTE_ROWS * 128;  // [SOL_ROUTE_ROWS]
  const int h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint4* kh = reinterpret_cast<const uint4*>(kmean + static_cast<int64_t>(h) * nb * 128);
  for (int i = tid; i < nb * 16; i += 256)
    *reinterpret_cast<uint4*>(ks + (i >> 4) * SOL_KEY_PAD + (i & 15) * 8) = kh[i];
  const int a0 = blockIdx.x * SOL_ROUTE_ROWS;
  for (int i = tid; i < SOL_ROUTE_ROWS * 32; i += 256) {
    const int r = i >> 5, a = a0 + r;
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    reinterpret_cast<float4*>(qs)[i] =
        a < nb ? reinterpret_cast<const float4*>(qmean + (static_cast<int64_t>(h) * nb + a) * 128)[i & 31]
               : z;
  }
  __syncthreads();
  const int rg = tid >> 4, cv = tid & 15;
  for (int pass = 0; pass < 2; ++pass) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    for (int b = rg; b < nb; b += 16) {
      const uint4 raw = *reinterpret_cast<const uint4*>(ks + b * SOL_KEY_PAD + cv * 8);
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
        if (pass == 0) {
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        } else {
          const float d0 = f.x - center[cv * 8 + 2 * e], d1 = f.y - center[cv * 8 + 2 * e + 1];
          acc[2 * e] += d0 * d0;
          acc[2 * e + 1] += d1 * d1;
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) part[rg * 128 + cv * 8 + e] = acc[e];
    __syncthreads();
    if (tid < 128) {
      float t = 0.0f;
      for (int r = 0; r < 16; ++r) t += part[r * 128 + tid];
      (pass == 0 ? center : var)[tid] = t / static_cast<float>(nb);
    }
    __syncthreads();
  }
  for (int r = warp; r < SOL_ROUTE_ROWS; r += 8) {
    const float* q = qs + r * 128;
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
    if (lane == 0) limit[r] = raw_mean * log2_scale + tau * sqrtf(variance + 1.0e-6f);
  }
  __syncthreads();
  const int r0 = (warp & 1) * 8;
  for (int w = warp >> 1; w < words; w += 4) {
    const int b = w * 32 + lane;
    const __half* kr = ks + min(b, nb - 1) * SOL_KEY_PAD;
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = 0.0f;
#pragma unroll 2
    for (int c = 0; c < 16; ++c) {
      const uint4 raw = *reinterpret_cast<const uint4*>(kr + c * 8);
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
        kf[2 * e] = f.x;
        kf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4 qa = reinterpret_cast<const float4*>(qs + (r0 + r) * 128 + c * 8)[0];
        const float4 qb = reinterpret_cast<const float4*>(qs + (r0 + r) * 128 + c * 8)[1];
        acc[r] = fmaf(qa.x, kf[0], acc[r]);
        acc[r] = fmaf(qa.y, kf[1], acc[r]);
        acc[r] = fmaf(qa.z, kf[2], acc[r]);
        acc[r] = fmaf(qa.w, kf[3], acc[r]);
        acc[r] = fmaf(qb.x, kf[4], acc[r]);
        acc[r] = fmaf(qb.y, kf[5], acc[r]);
        acc[r] = fmaf(qb.z, kf[6], acc[r]);
        acc[r] = fmaf(qb.w, kf[7], acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int a = a0 + r0 + r;
      const bool routed =
          b < nb && ((b >= a - 1 && b <= a + 1) || acc[r] * log2_scale > limit[r0 + r]);
      const uint32_t word = __ballot_sync(0xffffffffu, routed);
      if (lane == 0 && a < nb) bits[(static_cast<int64_t>(h) * nb + a) * words + w] = word;
    }
  }
}

// grid (CTAs per head, heads), 32 threads: the union of the routing rows of the CTA's query
// blocks (SOL_QBLOCKS c .. SOL_QBLOCKS c + SOL_QBLOCKS - 1) as an ascending block list and its
// length.
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

// Shared memory of sol_attention_kernel: two 128-row query tiles (the current work item's and the
// next one's), two 128-key K/V stages (one per key stream), the softmax exchange areas and
// barriers of the dense kernel, then two copies of the work item's routing words, block list
// and block count.
struct SolSmem {
  static constexpr int HALF = AttnSmem::HALF;
  static constexpr int Q_OFF = 0;                      // buffer b at Q_OFF + b * 2 * HALF
  static constexpr int KV_OFF = 4 * HALF;
  static constexpr int STAGE = 4 * HALF;
  static constexpr int X_OFF = KV_OFF + ATT_STAGES * STAGE;
  static constexpr int L_OFF = X_OFF + 2 * 2 * 2 * 128 * 4;
  static constexpr int BAR_OFF = L_OFF + 2 * 2 * 128 * 4;
  // q_full[2], q_empty[2], meta_full[2], meta_empty[2], kv_full[2], kv_empty[2], s_full[2],
  // p_full[2], o_done, drain, xbar[4][2][2], lbar[4]
  static constexpr int NBAR = 16 + 2 + 16 + 4;
  static constexpr int W_OFF = BAR_OFF + NBAR * 8 + 16;
  static constexpr int WORDS = SOL_QBLOCKS * SOL_MAX_WORDS;  // routing words of one item
  static constexpr int LIST_OFF = W_OFF + 2 * WORDS * 4;
  static constexpr int COUNT_OFF = LIST_OFF + 2 * SOL_MAX_WORDS * 32 * 4;
  static constexpr int TOTAL = COUNT_OFF + 16 + 1024;
};

// A persistent CTA per SM walks work items it = blockIdx.x, blockIdx.x + gridDim.x, ... (head
// it / ncta, query tile it % ncta: query blocks 2c and 2c + 1). An item is the tile against the
// ascending list of key blocks either of its query blocks routes, then the centroids. The stages
// (two 64-key blocks, or 128 centroids) alternate between two key streams, A taking stages
// 0, 2, 4, ... and B stages 1, 3, 5, ...: each stream has its own S and O in tensor memory and
// its own running row maxima and sums, so the MMA warp works on one stream while the softmax
// warps work on the other, and the epilogue merges the two streams by their row statistics.
// Stream t owns K/V slot t. Across items the ring and barrier phases run on (per-stream stage
// counts carried from item to item), the next item's Q tile, block list and first products are
// under way while the softmax warps finish the current item's epilogue, and the tensor memory
// is allocated once. The next item's first PV product overwrites O only after the softmax warps
// signal that item's first P, which they do after their epilogue has read O.
__global__ void __launch_bounds__(ATT_THREADS, 1)
    sol_attention_kernel(const __grid_constant__ CUtensorMap mq,
                         const __grid_constant__ CUtensorMap mk,
                         const __grid_constant__ CUtensorMap mv,
                         const __grid_constant__ CUtensorMap mkc,
                         const __grid_constant__ CUtensorMap mvc, const SolParams p) {
  using L = SolSmem;
  constexpr int D = 128;
  constexpr int NH = 2;
  constexpr int SUB = 64 * 128;  // one 64-row box of a 64-wide swizzled half: 8 KB
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;            // [buffer]
  uint64_t* q_empty = bars + 2;       // [buffer]
  uint64_t* meta_full = bars + 4;     // [buffer]
  uint64_t* meta_empty = bars + 6;    // [buffer]
  uint64_t* kv_full = bars + 8;       // [stream]
  uint64_t* kv_empty = bars + 10;     // [stream]
  uint64_t* s_full = bars + 12;       // [stream]
  uint64_t* p_full = bars + 14;       // [stream]
  uint64_t* o_done = bars + 16;
  uint64_t* drain = bars + 17;
  uint64_t* xbar = bars + 18;         // [quarter][stream][parity]
  uint64_t* lbar = xbar + 16;         // [quarter]
  float* xmax = reinterpret_cast<float*>(smem + L::X_OFF);
  float* xsum = reinterpret_cast<float*>(smem + L::L_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* rwords_all = reinterpret_cast<uint32_t*>(smem + L::W_OFF);  // [buffer][WORDS]
  int* slist_all = reinterpret_cast<int*>(smem + L::LIST_OFF);         // [buffer][512]
  int* mcount = reinterpret_cast<int*>(smem + L::COUNT_OFF);           // [buffer]

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  const int items = p.ncta * p.heads;
  const int ncent = (p.nb + 127) / 128;  // centroid stages

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&meta_full[i], 1);
      mbar_init(&meta_empty[i], 9);  // the eight softmax warps and the MMA warp
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
    tma_prefetch(&mkc);
    tma_prefetch(&mvc);
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
    // the work items' block lists and routing words (all lanes), Q tiles and K/V stages (lane 0)
    int kcount[2] = {0, 0};  // stages issued per stream, over all items
    int j = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++j) {
      const int buf = j & 1;
      const uint32_t use = static_cast<uint32_t>(j >> 1) & 1u;
      const int head = it / p.ncta, cta = it % p.ncta;
      if (!mbar_wait(&meta_empty[buf], use ^ 1u, abort_flag)) break;
      const int count = p.counts[head * p.ncta + cta];
      const int qb = cta * SOL_QBLOCKS + static_cast<int>(lane) / SOL_MAX_WORDS;
      const int w = static_cast<int>(lane) % SOL_MAX_WORDS;
      rwords_all[buf * L::WORDS + lane] =
          (qb < p.nb && w < p.words) ? p.bits[(static_cast<int64_t>(head) * p.nb + qb) * p.words + w]
                                     : 0u;
      const int* list = p.lists + (static_cast<int64_t>(head) * p.ncta + cta) * p.nb;
      for (int i = static_cast<int>(lane); i < count; i += 32) slist_all[buf * 512 + i] = list[i];
      if (lane == 0) mcount[buf] = count;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&meta_full[buf]);
        if (!mbar_wait(&q_empty[buf], use ^ 1u, abort_flag)) {
          *abort_flag = 1;
        } else {
          uint8_t* sq = smem + L::Q_OFF + buf * 2 * L::HALF;
          mbar_expect_tx(&q_full[buf], NH * L::HALF);
          tma_load_4d(sq, &mq, &q_full[buf], 0, cta * 128, head, 0);
          tma_load_4d(sq + L::HALF, &mq, &q_full[buf], 64, cta * 128, head, 0);
          const int* sl = slist_all + buf * 512;
          const int ns = (count + 1) / 2;
          const int nst = ns + ncent;
          for (int i = 0; i < nst; ++i) {
            const int t = i & 1;
            const uint32_t parity = static_cast<uint32_t>(kcount[t]) & 1u;
            if (!mbar_wait(&kv_empty[t], parity ^ 1u, abort_flag)) break;
            ++kcount[t];
            uint8_t* sk = smem + L::KV_OFF + t * L::STAGE;
            uint8_t* sv = sk + 2 * L::HALF;
            mbar_expect_tx(&kv_full[t], 2 * NH * L::HALF);
            if (i < ns) {
              const int kb0 = sl[2 * i];
              const int kb1 = 2 * i + 1 < count ? sl[2 * i + 1] : kb0;  // a masked stand-in
#pragma unroll
              for (int h2 = 0; h2 < NH; ++h2) {
                tma_load_4d(sk + h2 * L::HALF, &mk, &kv_full[t], h2 * 64, kb0 * 64, head, 0);
                tma_load_4d(sk + h2 * L::HALF + SUB, &mk, &kv_full[t], h2 * 64, kb1 * 64, head, 0);
                tma_load_4d(sv + h2 * L::HALF, &mv, &kv_full[t], h2 * 64, kb0 * 64, head, 0);
                tma_load_4d(sv + h2 * L::HALF + SUB, &mv, &kv_full[t], h2 * 64, kb1 * 64, head, 0);
              }
            } else {
              const int c0 = (i - ns) * 128;
#pragma unroll
              for (int h2 = 0; h2 < NH; ++h2) {
                tma_load_3d(sk + h2 * L::HALF, &mkc, &kv_full[t], h2 * 64, c0, head);
                tma_load_3d(sk + h2 * L::HALF + SUB, &mkc, &kv_full[t], h2 * 64, c0 + 64, head);
                tma_load_3d(sv + h2 * L::HALF, &mvc, &kv_full[t], h2 * 64, c0, head);
                tma_load_3d(sv + h2 * L::HALF + SUB, &mvc, &kv_full[t], h2 * 64, c0 + 64, head);
              }
            }
          }
        }
      }
      __syncwarp();
      if (*abort_flag) break;
    }
    if (lane == 0 && *abort_flag) {
      // after a timeout, give copies still in flight a bounded moment to land
      const uint64_t t0 = global_ns();
      while (global_ns() - t0 < 100000000ull) {
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(ATT_BM, ATT_BN);
      constexpr uint32_t idesc_o = idesc_f16(ATT_BM, D) | (1u << 16);  // B (V) MN-major
      int fk[2] = {0, 0};  // K/V stages consumed per stream, over all items
      int pk[2] = {0, 0};  // P signals consumed per stream
      bool ok = true;
      int j = 0;
      for (int it = blockIdx.x; ok && it < items; it += gridDim.x, ++j) {
        const int buf = j & 1;
        const uint32_t use = static_cast<uint32_t>(j >> 1) & 1u;
        if (!mbar_wait(&meta_full[buf], use, abort_flag)) break;
        const int count = mcount[buf];
        mbar_arrive(&meta_empty[buf]);
        const int nst = (count + 1) / 2 + ncent;
        if (!mbar_wait(&q_full[buf], use, abort_flag)) break;
        const uint32_t sq = smem_u32(smem + L::Q_OFF + buf * 2 * L::HALF);
        auto s_mma = [&](int t) {  // S_t = Q K^T of the stage in slot t
          const uint32_t sk = smem_u32(smem + L::KV_OFF + t * L::STAGE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * L::HALF + (kk & 3) * 32;
            umma_bf16(tmem + t * 128, sdesc_k128(sq + off), sdesc_k128(sk + off), idesc_s,
                      kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[t]);
        };
        auto pv_mma = [&](int t, bool first) {  // O_t += P_t V of the stage in slot t
          const uint32_t sv = smem_u32(smem + L::KV_OFF + t * L::STAGE + 2 * L::HALF);
#pragma unroll
          for (int kk = 0; kk < ATT_BN / 16; ++kk) {
            umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8 + (kk >= 4 ? 32 : 0),
                         sdesc_mn128(sv + kk * 2048, L::HALF), idesc_o,
                         (!first || kk > 0) ? 1u : 0u);
          }
        };
        auto next_kv = [&](int t) {
          const bool got = mbar_wait(&kv_full[t], static_cast<uint32_t>(fk[t]) & 1u, abort_flag);
          ++fk[t];
          if (got) tc_fence_after();
          return got;
        };
        for (int t = 0; ok && t < 2 && t < nst; ++t) {
          ok = next_kv(t);
          if (ok) s_mma(t);
        }
        for (int k = 0; ok && 2 * k < nst; ++k) {
          for (int t = 0; t < 2 && ok; ++t) {
            const int i = 2 * k + t;
            if (i >= nst) break;
            if (!mbar_wait(&p_full[t], static_cast<uint32_t>(pk[t]) & 1u, abort_flag)) {
              ok = false;
              break;
            }
            ++pk[t];
            tc_fence_after();
            pv_mma(t, k == 0);
            umma_commit(&kv_empty[t]);
            if (i + 2 < nst) {
              ok = next_kv(t);
              if (ok) s_mma(t);
            }
          }
        }
        if (!ok) break;
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
    int sk[2] = {0, 0};  // stages seen per stream, over all items (barrier and buffer phases)
    bool ok = true;
    int j = 0;
    for (int it = blockIdx.x; ok && it < items; it += gridDim.x, ++j) {
      const int buf = j & 1;
      const uint32_t use = static_cast<uint32_t>(j >> 1) & 1u;
      const int head = it / p.ncta, cta = it % p.ncta;
      const int row0 = cta * 128;
      if (!mbar_wait(&meta_full[buf], use, abort_flag)) break;
      const int count = mcount[buf];
      const int* slist = slist_all + buf * 512;
      const uint32_t* rw = rwords_all + buf * L::WORDS + (row >> 6) * SOL_MAX_WORDS;
      const int ns = (count + 1) / 2;  // exact stages: two 64-key blocks each
      const int nst = ns + ncent;      // then the centroid stages
      float m_run[2] = {-INFINITY, -INFINITY};
      float l_run[2] = {0.0f, 0.0f};
      // stage i (the k-th of stream t in this item, g-th over all items) for this warp's 64 keys:
      // an exact block kb (or none) or centroids c0 .. c0 + 63; instantiated once per kind so
      // each loop's body stays compact
      auto stage = [&](const int i, const int t, const int k, auto kind) {
        constexpr bool exact = decltype(kind)::value;
        const int g = sk[t]++;
        int kb = -1, nk = 0, c0 = 0;
        if constexpr (exact) {
          const int li = 2 * i + half;
          kb = li < count ? slist[li] : -1;
          nk = kb >= 0 ? min(SOL_BLOCK, p.tokens - kb * SOL_BLOCK) : 0;
        } else {
          c0 = (i - ns) * 128 + half * 64;
        }
        if (!mbar_wait(&s_full[t], static_cast<uint32_t>(g) & 1u, abort_flag)) {
          ok = false;
          return;
        }
        tc_fence_after();
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
              for (int jj = 0; jj < 32; ++jj)
                if (c * 32 + jj >= nk) sr[c][jj] = __float_as_uint(-1.0e30f);
          }
        } else {
          const int w0 = c0 >> 5;
          const uint32_t words[2] = {w0 < p.words ? rw[w0] : ~0u,
                                     w0 + 1 < p.words ? rw[w0 + 1] : ~0u};
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const int b = c0 + c * 32 + jj;
              const float bias = b == p.nb - 1 ? p.last_log2 : 6.0f;
              const bool take = b < p.nb && !((words[c] >> jj) & 1u);
              sr[c][jj] = __float_as_uint(take ? fmaf(__uint_as_float(sr[c][jj]), sl2, bias)
                                               : -INFINITY);
            }
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
        if constexpr (exact)
          mine = routed_row ? raw * sl2 : -INFINITY;
        else
          mine = raw;
        float* xm = xmax + (t * 2 + (g & 1)) * 256;
        xm[half * 128 + row] = mine;
        uint64_t* xb = &xbar[(quarter * 2 + t) * 2 + (g & 1)];
        mbar_arrive(xb);
        if (!mbar_wait(xb, static_cast<uint32_t>(g >> 1) & 1u, abort_flag)) {
          ok = false;
          return;
        }
        const float m_blk = fmaxf(mine, xm[(1 - half) * 128 + row]);
        float alpha = 1.0f;
        bool rescale = false;
        if (k > 0) {
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
        // an exact block is routed or not for a whole warp (its 32 rows lie in one query block):
        // a warp that does not route it writes P = 0 without exponentials
        if (!exact || routed_row) {
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
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            tmem_ld32(o_col + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) o[jj] = __float_as_uint(__uint_as_float(o[jj]) * alpha);
            tmem_st32(o_col + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      };
      // the exact stages, then the centroid stages, each alternating between the streams
      for (int i = 0; i < ns && ok; ++i) stage(i, i & 1, i >> 1, std::true_type{});
      for (int i = ns; i < nst && ok; ++i) stage(i, i & 1, i >> 1, std::false_type{});
      if (!ok) break;
      if (lane == 0) mbar_arrive(&meta_empty[buf]);  // done with the item's words and list
      for (int t = 0; t < 2; ++t) xsum[(t * 2 + half) * 128 + row] = l_run[t];
      mbar_arrive(&lbar[quarter]);
      if (!mbar_wait(&lbar[quarter], static_cast<uint32_t>(j) & 1u, abort_flag) ||
          !mbar_wait(o_done, static_cast<uint32_t>(j) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int tok = row0 + row;
      bool store = tok < p.tokens;
      // merge the streams: O = (O_A 2^(m_A - m) + O_B 2^(m_B - m)) / (l_A 2^(m_A - m) + ...)
      const float la = l_run[0] + xsum[(0 * 2 + 1 - half) * 128 + row];
      const float lb = l_run[1] + xsum[(1 * 2 + 1 - half) * 128 + row];
      const float m = fmaxf(m_run[0], m_run[1]);
      const bool has_b = nst > 1;
      const float sa = m_run[0] == -INFINITY ? 0.0f : ex2_approx(m_run[0] - m);
      const float sb = (!has_b || m_run[1] == -INFINITY) ? 0.0f : ex2_approx(m_run[1] - m);
      const float inv_l = 1.0f / (la * sa + lb * sb);
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
      auto fin = [&](uint32_t ra, uint32_t rb) -> float {
        const float o = (__uint_as_float(ra) * sa + (has_b ? __uint_as_float(rb) * sb : 0.0f)) * inv_l;
        if (p.gate == nullptr) return o;
        const float r = p.out_f16 ? __half2float(__float2half_rn(o)) : bf16_round(o);
        return r * gv;
      };
      const uint32_t oa_col = tmem + lane_base + 256 + half * (D / 2);
      const uint32_t ob_col = oa_col + 128;
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) {
        uint32_t oa[32], ob[32];
        tmem_ld32(oa_col + c * 32, oa);
        tmem_ld32(ob_col + c * 32, ob);
        tmem_wait_ld();
        if (store) {
          uint8_t* base = static_cast<uint8_t*>(p.out) +
                          (dst_row * p.ld_out + head * D + half * (D / 2) + c * 32) * 2;
          uint32_t w16[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float o0 = fin(oa[2 * e], ob[2 * e]), o1 = fin(oa[2 * e + 1], ob[2 * e + 1]);
            w16[e] = p.out_f16 ? pack_f16x2(o0, o1) : pack_bf16x2(o0, o1);
          }
          store_row32(reinterpret_cast<__nv_bfloat16*>(base), w16, 32);
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
