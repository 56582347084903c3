// 3x3x3 video-VAE convolution as an implicit GEMM on tcgen05, channels-last (F, H, W, C).
//
//   out[f, h, w, n] = sum_{kt, kh, kw, c} xpad[f + kt, h + kh, w + kw, c] * weight[n, kt, kh, kw, c]
//
// Restates Conv3dBlock (kinomlx/models/ltx2/video_vae/blocks.py:97-139): temporal replicate
// padding (causal: two copies of the first frame; otherwise one at each end), spatial zero
// padding of one, fp32 accumulation rounded to bf16, then the bias added in bf16, and optionally
// the residual added in bf16 (blocks.py:165-169). The weight is the reference's OTHWI layout,
// i.e. an (N, 27 * Cin) K-major matrix.
//
// GEMM view: M = output voxels, N = output channels, K = 27 * Cin. An M tile is a box of
// tf x th x tw voxels (128 in all). For each K block (one tap (kt, kh, kw), 64 channels) the TMA
// producer loads the shifted input box of every frame of the tile straight from the unpadded
// tensor: spatial padding is the TMA's zero fill at out-of-range coordinates (the channel
// coordinate stays 64-aligned), temporal replicate padding is a clamp of the frame coordinate.
// No im2col buffer, no padded copy. The MMA and epilogue roles are the GEMM's.
//
// Epilogue store modes: plain (same geometry), or depth-to-space (decoder.py:80-121): the
// weight rows are reordered on the host to sub-position-major order (n = sub * C' + c), so a
// 32-column chunk is 32 channels of one destination voxel; the first output frame is dropped
// when the temporal stride is 2.
#pragma once
#include "kino_common.cuh"
#include "kino_gemm.cuh"

namespace kino {

struct ConvShape {
  int F, H, W, Cin, N;
  int tf, th, tw;
  int fb, hb, wb;
  int boxes;  // fb * hb * wb voxel boxes of 128
  int tiles_m, tiles_n, num_tiles, kblocks, cblocks;  // an M tile is MT consecutive boxes
  int splits, kper;  // split-K: num_tiles = tiles_m * tiles_n * splits, kper K blocks per split
  int pad_front;
  int st, sh, sw, drop;  // depth-to-space strides (1,1,1,0 = plain store)
  int Fo, Ho, Wo, Co;    // output geometry
};

struct ConvEpi {
  const __nv_bfloat16* bias;      // [N] (in the same row order as the weight) or null
  const __nv_bfloat16* residual;  // plain mode only: same geometry as the output, or null
  // GroupNorm(32) statistics of the stored output (the next layer's norm), or null: every
  // epilogue warp keeps, in lane g, the count, mean and sum of squared deviations of group g
  // over the values it stored (merged chunk by chunk with Chan's pairwise formula) and writes
  // them as one record per lane quarter (CTA * 4 + quarter); CTA 0 writes the record count
  // into the header.
  float* stats;
  int group_size;  // output channels per group (output channels / 32)
  // Split-K (single-SM kernel, MT = 1): int arrival counters, one per output tile (zero between
  // launches), and the fp32 partial accumulators [tile][split][128 rows][BN].
  int* split_count;
  float* split_partial;
};

// GroupNorm statistics layout (floats): [0] record count (int), [4, 36) mean, [36, 68) rstd,
// record r at GN_STATS_RECORDS + r * 96: (count, mean, m2) for each of the 32 groups.
constexpr int GN_STATS_RECORDS = 128;

// (n_a, mean_a, m2_a) <- merge with (n_b, mean_b, m2_b) (Chan, Golub & LeVeque).
__device__ __forceinline__ void chan_merge(float& na, float& ma, float& m2a, float nb, float mb,
                                           float m2b) {
  if (nb <= 0.0f) return;
  const float n = na + nb;
  const float delta = mb - ma;
  ma += delta * (nb / n);
  m2a += m2b + delta * delta * (na * nb / n);
  na = n;
}

// GroupNorm statistics of one 32-channel chunk (groups of GS channels) over a warp's 32 voxels
// (the live ones): count, mean and m2 per group, merged into the lane that owns the group.
template <int GS>
__device__ __forceinline__ void conv_chunk_stats(const float (&v)[32], bool live, int first,
                                                 uint32_t lane, float& n, float& mean,
                                                 float& m2) {
  const float cnt = __popc(__ballot_sync(0xffffffffu, live)) * static_cast<float>(GS);
  if (cnt <= 0.0f) return;
#pragma unroll
  for (int k0 = 0; k0 < 32; k0 += GS) {
    float s1 = 0.0f;
#pragma unroll
    for (int j = 0; j < GS; ++j) s1 += v[k0 + j];
    const float mean_c = warp_sum_f(live ? s1 : 0.0f) / cnt;
    float d2 = 0.0f;
#pragma unroll
    for (int j = 0; j < GS; ++j) {
      const float dv = v[k0 + j] - mean_c;
      d2 = fmaf(dv, dv, d2);
    }
    const float m2_c = warp_sum_f(live ? d2 : 0.0f);
    if (static_cast<int>(lane) == first + k0 / GS) chan_merge(n, mean, m2, cnt, mean_c, m2_c);
  }
}

// Epilogue of one 128-voxel box of an M tile: thread `m` (its voxel) reads the accumulator
// columns of 32-column chunks [c_begin, c_end) at taddr, adds bias and residual, stores (plain or
// depth-to-space) and gathers the GroupNorm statistics of what it stored.
template <int BN>
__device__ __forceinline__ void conv_store_box(const ConvShape& s, const ConvEpi& e,
                                               __nv_bfloat16* __restrict__ out, int box, int nt,
                                               uint32_t taddr, int m, uint32_t lane,
                                               float& gn_n, float& gn_mean, float& gn_m2,
                                               int c_begin = 0, int c_end = BN / 32,
                                               const float* psum = nullptr, int splits = 0) {
  const int box_rows = s.th * s.tw;
  const int cpo = s.Co;  // channels per output voxel
  const int wbi = box % s.wb;
  const int hbi = (box / s.wb) % s.hb;
  const int fbi = box / (s.wb * s.hb);
  const int wi = m % s.tw, hi = (m / s.tw) % s.th, fi = m / box_rows;
  const int f = fbi * s.tf + fi, h = hbi * s.th + hi, w = wbi * s.tw + wi;
  const bool valid = f < s.F && h < s.H && w < s.W;
#pragma unroll 1
  for (int c = c_begin; c < c_end; ++c) {
    const int n0 = nt * BN + c * 32;
    if (n0 >= s.N) break;  // warp-uniform
    // destination voxel and channel offset of this 32-column chunk
    const int sub = n0 / cpo;
    const int ch0 = n0 - sub * cpo;
    const int a = sub / (s.sh * s.sw), bb = (sub / s.sw) % s.sh, ee = sub % s.sw;
    const int fo = f * s.st + a - s.drop, ho = h * s.sh + bb, wo = w * s.sw + ee;
    const bool live = valid && fo >= 0 && fo < s.Fo;
    const int64_t off =
        live ? ((static_cast<int64_t>(fo) * s.Ho + ho) * s.Wo + wo) * cpo + ch0 : 0;
    // the chunk's residual loads go out before the accumulator read, so their latencies overlap
    uint4 res[4];
    const bool use_res = e.residual != nullptr && live;
#pragma unroll
    for (int g = 0; g < 4; ++g)
      res[g] = (use_res && n0 + g * 8 < s.N)
                   ? *reinterpret_cast<const uint4*>(e.residual + off + g * 8)
                   : make_uint4(0u, 0u, 0u, 0u);
    uint32_t r[32];
    if (psum == nullptr) {
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
    } else {
      // split-K: the splits' fp32 partial sums of this row, added in split order (the same
      // order whichever CTA finishes last, so the result does not depend on timing)
      float acc32[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc32[j] = 0.0f;
      for (int ks = 0; ks < splits; ++ks) {
        const float4* src =
            reinterpret_cast<const float4*>(psum + (static_cast<int64_t>(ks) * 128 + m) * BN + c * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 f4 = __ldcg(src + q);
          acc32[4 * q] += f4.x;
          acc32[4 * q + 1] += f4.y;
          acc32[4 * q + 2] += f4.z;
          acc32[4 * q + 3] += f4.w;
        }
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(acc32[j]);
    }
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = bf16_round(__uint_as_float(r[j]));
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (n0 + g * 8 < s.N) {
        float add[8];
        if (e.bias != nullptr) {
          const uint4 raw = *reinterpret_cast<const uint4*>(e.bias + n0 + g * 8);
          const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 fb = unpack_bf16x2(w4[q]);
            add[2 * q] = fb.x;
            add[2 * q + 1] = fb.y;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) v[g * 8 + j] = bf16_round(v[g * 8 + j] + add[j]);
        }
        if (use_res) {
          const uint32_t w4[4] = {res[g].x, res[g].y, res[g].z, res[g].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 fr = unpack_bf16x2(w4[q]);
            v[g * 8 + 2 * q] += fr.x;
            v[g * 8 + 2 * q + 1] += fr.y;
          }
        }
      }
    }
    if (live) {
      uint32_t o16[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) o16[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
      store_row32(out + off, o16, s.N - n0);
    }
    if (e.stats != nullptr) {
      // the stored (bf16) values of this chunk, group by group: the warp's 32 voxels give
      // one (count, mean, m2) per group, merged into the lane that owns the group
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
      const int first = ch0 / e.group_size;
      switch (e.group_size) {
        case 1: conv_chunk_stats<1>(v, live, first, lane, gn_n, gn_mean, gn_m2); break;
        case 2: conv_chunk_stats<2>(v, live, first, lane, gn_n, gn_mean, gn_m2); break;
        case 4: conv_chunk_stats<4>(v, live, first, lane, gn_n, gn_mean, gn_m2); break;
        case 8: conv_chunk_stats<8>(v, live, first, lane, gn_n, gn_mean, gn_m2); break;
        case 16: conv_chunk_stats<16>(v, live, first, lane, gn_n, gn_mean, gn_m2); break;
        default: conv_chunk_stats<32>(v, live, first, lane, gn_n, gn_mean, gn_m2); break;
      }
    }
  }
}

// Shared memory of a conv tile of MT voxel boxes: per stage MT A boxes (128 x 64 each) and one
// weight block (BN x 64) that all of them use.
template <int BN, int STAGES, int MT>
struct ConvSmem {
  static constexpr int A1_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int A_BYTES = MT * A1_BYTES;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int TOTAL = TILE_BYTES + BAR_BYTES + 1024;
};

// MT > 1 (narrow outputs, BN = 128): MT boxes share each weight block, so the tile's operand
// traffic per tensor-core cycle falls from 2 to (MT + 1) / MT blocks of 16 KB per 128 x 128 x 64.
template <int BN, int STAGES, int MT>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    conv3d_tc_kernel(const __grid_constant__ CUtensorMap map_x,
                     const __grid_constant__ CUtensorMap map_w, __nv_bfloat16* __restrict__ out,
                     const ConvShape s, const ConvEpi e) {
  using L = ConvSmem<BN, STAGES, MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::TILE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&map_x);
    tma_prefetch(&map_w);
  }
  griddep_wait();  // the previous kernel has finished with its memory and tensor memory
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, 2 * MT * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  griddep_launch();
  const int box_rows = s.th * s.tw;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < s.num_tiles; t += gridDim.x) {
        const int tile = t % (s.tiles_m * s.tiles_n);
        const int mt = tile % s.tiles_m;
        const int nt = tile / s.tiles_m;
        const int kb_begin = (t / (s.tiles_m * s.tiles_n)) * s.kper;
        const int kb_end = kb_begin + s.kper < s.kblocks ? kb_begin + s.kper : s.kblocks;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          const int tap = kb / s.cblocks;
          const int cb = kb - tap * s.cblocks;
          const int kt = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
          uint8_t* sa = smem + stage * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          mbar_expect_tx(&full[stage], L::STAGE_BYTES);
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            const int box = mt * MT + i;
            const int wbi = box % s.wb;
            const int hbi = (box / s.wb) % s.hb;
            const int fbi = box / (s.wb * s.hb);
            // a box past the last one loads zero fill (width coordinate out of range)
            const int f0 = fbi * s.tf, h0 = hbi * s.th;
            const int w0 = box < s.boxes ? wbi * s.tw : s.W + 64;
            for (int fi = 0; fi < s.tf; ++fi) {
              int fs = f0 + fi + kt - s.pad_front;
              fs = fs < 0 ? 0 : (fs > s.F - 1 ? s.F - 1 : fs);
              tma_load_4d(sa + i * L::A1_BYTES + fi * box_rows * 128, &map_x, &full[stage],
                          cb * 64, w0 + kw - 1, h0 + kh - 1, fs);
            }
          }
          tma_load_2d(sb, &map_w, &full[stage], kb * GEMM_BK, nt * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      if (*abort_flag) {
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--stage < 0) {
            stage = STAGES - 1;
            phase ^= 1u;
          }
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(&full[stage], phase) && global_ns() - t0 < 200000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(GEMM_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < s.num_tiles; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * MT * BN;
        bool ok = true;
        const int kb_begin = (t / (s.tiles_m * s.tiles_n)) * s.kper;
        const int kb_end = kb_begin + s.kper < s.kblocks ? kb_begin + s.kper : s.kblocks;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int i = 0; i < MT; ++i) {
#pragma unroll
            for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
              umma_bf16(d_tmem + i * BN, sdesc_k128(sa + i * L::A1_BYTES + kk * 32),
                        sdesc_k128(sb + kk * 32), idesc, (kb > kb_begin || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      umma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 200000000ull) {
      }
    }
  } else {
    const int quarter = warp & 3;
    const int m = quarter * 32 + static_cast<int>(lane);
    float gn_n = 0.0f, gn_mean = 0.0f, gn_m2 = 0.0f;  // statistics of group `lane`
    int local = 0;
    for (int t = blockIdx.x; t < s.num_tiles; t += gridDim.x, ++local) {
      const int tile = t % (s.tiles_m * s.tiles_n);
      const int mt = tile % s.tiles_m;
      const int nt = tile / s.tiles_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
      tc_fence_after();
      if (MT == 1 && s.splits > 1) {
        // split-K: store this split's fp32 accumulators, free the TMEM buffer, and let the CTA
        // that completes the tile's last split run the epilogue over all partial sums
        const int ks = t / (s.tiles_m * s.tiles_n);
        float* part = e.split_partial + static_cast<int64_t>(tile) * s.splits * 128 * BN;
        const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + acc * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(part + (static_cast<int64_t>(ks) * 128 + m) * BN + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(dst + q, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                        __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        // Each warp owns its 32 rows: its partial rows are out (fence) before its counter
        // (tile, lane quarter) moves; the warp that brings the counter to `splits` sums them.
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          int* cnt = e.split_count + tile * 4 + quarter;
          const int prev = atomicAdd(cnt, 1);
          last = prev == s.splits - 1;
          if (last) atomicExch(cnt, 0);  // ready for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          if (mt < s.boxes)
            conv_store_box<BN>(s, e, out, mt, nt, 0u, m, lane, gn_n, gn_mean, gn_m2, 0, BN / 32,
                               part, s.splits);
        }
        continue;
      }
#pragma unroll 1
      for (int bi = 0; bi < MT; ++bi) {
        const int box = mt * MT + bi;
        if (box >= s.boxes) break;  // warp-uniform
        conv_store_box<BN>(s, e, out, box, nt,
                           tmem_base + ((quarter * 32) << 16) + acc * MT * BN + bi * BN, m, lane,
                           gn_n, gn_mean, gn_m2);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (e.stats != nullptr) {
      float* rec = e.stats + GN_STATS_RECORDS + (blockIdx.x * 4 + quarter) * 96 + lane * 3;
      rec[0] = gn_n;
      rec[1] = gn_mean;
      rec[2] = gn_m2;
      if (blockIdx.x == 0 && warp == 2 && lane == 0)
        *reinterpret_cast<int*>(e.stats) = static_cast<int>(gridDim.x) * 4;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * MT * BN);
  }
}

// ----------------------------------------------------------------------------- CTA pairs
// The same convolution on CTA pairs (cluster of 2): a pair tile is two consecutive voxel boxes
// (one per CTA, M = 256) by BN output channels, issued by the even CTA as
// tcgen05.mma.cta_group::2. Each CTA loads its own box and BN / 2 of the weight rows, so the
// per-SM operand traffic per tensor-core cycle is three quarters (BN = 256) or a little over
// half (BN = 128) of the single-CTA tile's. TMA loads complete on the even CTA's barriers (no
// multicast loads); MMA completion is committed to both CTAs; each CTA stores its own box.
// A stage holds KSUB consecutive K blocks (each: this CTA's box and its half of the weight
// rows), so that one barrier round trip covers KSUB x 4 MMAs: with BN = 128 an MMA is only 64
// tensor cycles and the per-stage wait would otherwise show between the groups.
// HALO (input rows loaded once for three taps):
//   1 (along W) the box is one 128-voxel row and a K sub-block one (kt, kh, channel block)
//     triple: its input row is loaded with a voxel of halo on each side (130 rows) and serves the
//     kw = 0, 1, 2 taps as A operands starting 0, 1 and 2 rows in;
//   2 (along H) the box is th rows of tw voxels of one frame and a K sub-block one (kt, kw,
//     channel block) triple: th + 2 input rows (a row of halo above and below) serve the
//     kh = 0, 1, 2 taps as A operands starting 0, tw and 2 tw rows in (whole 1024-byte swizzle
//     atoms, tw >= 8);
//   each tap with its own weight block, so the input crosses from L2 9 times per voxel instead
//   of 27. The 128-byte swizzle is a function of the absolute shared-memory address (measured:
//   the MMA reads the TMA's swizzled rows correctly from a start 1 or 2 rows into a 1024-byte
//   atom with the descriptor's base-offset field left at 0, and wrongly with it set to the row
//   phase), so the shifted operands are plain descriptors of the shifted addresses.
constexpr int CONV_HALO_ROWS = GEMM_BM + 2;
template <int BN, int STAGES, int KSUB, int HALO = 0>
struct ConvPairSmem {
  // this CTA's input: a box, a halo row (130 rows), or th + 2 rows of tw (at most 6 x 32)
  static constexpr int A_BYTES = HALO == 1 ? 17 * 1024 : (HALO == 2 ? 24 * 1024 : GEMM_BM * GEMM_BK * 2);
  static constexpr int B1_BYTES = (BN / 2) * GEMM_BK * 2;  // this CTA's half of one tap's weights
  static constexpr int B_BYTES = (HALO ? 3 : 1) * B1_BYTES;
  static constexpr int SUB_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = KSUB * SUB_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int XCH_BYTES = 4 * 32 * 3 * 4;  // GroupNorm statistics handed between halves
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int TOTAL = TILE_BYTES + XCH_BYTES + BAR_BYTES + 1024;
};

template <int BN, int STAGES, int KSUB, int HALO = 0>
__global__ void __launch_bounds__(CONV_PAIR_THREADS, 1)
    conv3d_2sm_kernel(const __grid_constant__ CUtensorMap map_x,
                      const __grid_constant__ CUtensorMap map_w, __nv_bfloat16* __restrict__ out,
                      const ConvShape s, const ConvEpi e) {
  using L = ConvPairSmem<BN, STAGES, KSUB, HALO>;
  // K sub-blocks: one per (tap, channel block), or per (kt, kh | kw, channel block) with HALO
  const int ksub_blocks = HALO ? 9 * s.cblocks : s.kblocks;
  // bytes the TMA delivers per sub-block
  const int a_tx = HALO == 1 ? CONV_HALO_ROWS * 128
                             : (HALO == 2 ? (s.th + 2) * s.tw * 128 : L::A_BYTES);
  const int sub_tx = a_tx + L::B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* stats_xch = reinterpret_cast<float*>(smem + L::TILE_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::TILE_BYTES + L::XCH_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_rank();  // 0: leader (issues the MMAs), 1: peer
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * CONV_PAIR_EPI_WARPS);  // the epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&map_x);
    tma_prefetch(&map_w);
  }
  griddep_wait();  // the previous kernel has finished with its memory and tensor memory
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive or complete_tx
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  griddep_launch();
  const int box_rows = s.th * s.tw;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = pair; t < s.num_tiles; t += pairs) {
        const int mt = t % s.tiles_m;
        const int nt = t / s.tiles_m;
        const int box = mt * 2 + static_cast<int>(rank);
        const int wbi = box % s.wb;
        const int hbi = (box / s.wb) % s.hb;
        const int fbi = box / (s.wb * s.hb);
        // a box past the last one loads zero fill (width coordinate out of range)
        const int f0 = fbi * s.tf, h0 = hbi * s.th;
        const int w0 = box < s.boxes ? wbi * s.tw : s.W + 64;
        for (int kb0 = 0; kb0 < ksub_blocks; kb0 += KSUB) {
          const int nsub = ksub_blocks - kb0 < KSUB ? ksub_blocks - kb0 : KSUB;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
          const uint32_t leader_full = smem_u32(&full[stage]) & kPairLeaderMask;
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * nsub * sub_tx);
          for (int j = 0; j < nsub; ++j) {
            const int kb = kb0 + j;
            uint8_t* sa = smem + stage * L::STAGE_BYTES + j * L::SUB_BYTES;
            uint8_t* sb = sa + L::A_BYTES;
            if constexpr (HALO == 2) {
              // rows h0 - 1 .. h0 + th of frame f0 + kt, columns shifted by kw (tf = 1)
              const int tri = kb / s.cblocks;
              const int cb = kb - tri * s.cblocks;
              const int kt = tri / 3, kw = tri % 3;
              int fs = f0 + kt - s.pad_front;
              fs = fs < 0 ? 0 : (fs > s.F - 1 ? s.F - 1 : fs);
              tma_load_4d_pair(sa, &map_x, leader_full, cb * 64, w0 + kw - 1, h0 - 1, fs);
#pragma unroll
              for (int kh = 0; kh < 3; ++kh)
                tma_load_2d_pair(sb + kh * L::B1_BYTES, &map_w, leader_full,
                                 ((kt * 9 + kh * 3 + kw) * s.cblocks + cb) * GEMM_BK,
                                 nt * BN + static_cast<int>(rank) * (BN / 2));
            } else if constexpr (HALO == 1) {
              // the row w0 - 1 .. w0 + 128 of frame f0 + kt, row h0 + kh (tf = th = 1)
              const int tri = kb / s.cblocks;
              const int cb = kb - tri * s.cblocks;
              const int kt = tri / 3, kh = tri % 3;
              int fs = f0 + kt - s.pad_front;
              fs = fs < 0 ? 0 : (fs > s.F - 1 ? s.F - 1 : fs);
              tma_load_4d_pair(sa, &map_x, leader_full, cb * 64, w0 - 1, h0 + kh - 1, fs);
#pragma unroll
              for (int kw = 0; kw < 3; ++kw)
                tma_load_2d_pair(sb + kw * L::B1_BYTES, &map_w, leader_full,
                                 ((kt * 9 + kh * 3 + kw) * s.cblocks + cb) * GEMM_BK,
                                 nt * BN + static_cast<int>(rank) * (BN / 2));
            } else {
              const int tap = kb / s.cblocks;
              const int cb = kb - tap * s.cblocks;
              const int kt = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
              for (int fi = 0; fi < s.tf; ++fi) {
                int fs = f0 + fi + kt - s.pad_front;
                fs = fs < 0 ? 0 : (fs > s.F - 1 ? s.F - 1 : fs);
                tma_load_4d_pair(sa + fi * box_rows * 128, &map_x, leader_full, cb * 64,
                                 w0 + kw - 1, h0 + kh - 1, fs);
              }
              tma_load_2d_pair(sb, &map_w, leader_full, kb * GEMM_BK,
                               nt * BN + static_cast<int>(rank) * (BN / 2));
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // After a timeout, give loads still in flight a bounded moment to land.
      if (*abort_flag && issued > 0) {
        const uint64_t t0 = global_ns();
        while (global_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16(256, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = pair; t < s.num_tiles; t += pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb0 = 0; kb0 < ksub_blocks; kb0 += KSUB) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
            if (kb0 + j < ksub_blocks) {
              const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES + j * L::SUB_BYTES);
              const uint32_t sb = sa + L::A_BYTES;
              if constexpr (HALO == 2) {
                const uint32_t pitch = static_cast<uint32_t>(s.tw) * 128;  // one input row
#pragma unroll
                for (int kh = 0; kh < 3; ++kh) {
#pragma unroll
                  for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
                    umma_bf16_pair(d_tmem, sdesc_k128(sa + kh * pitch + kk * 32),
                                   sdesc_k128(sb + kh * L::B1_BYTES + kk * 32), idesc,
                                   (kb0 + j > 0 || kh > 0 || kk > 0) ? 1u : 0u);
                  }
                }
              } else if constexpr (HALO == 1) {
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
#pragma unroll
                  for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
                    umma_bf16_pair(d_tmem, sdesc_k128(sa + kw * 128 + kk * 32),
                                   sdesc_k128(sb + kw * L::B1_BYTES + kk * 32), idesc,
                                   (kb0 + j > 0 || kw > 0 || kk > 0) ? 1u : 0u);
                  }
                }
              } else {
#pragma unroll
                for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
                  umma_bf16_pair(d_tmem, sdesc_k128(sa + kk * 32), sdesc_k128(sb + kk * 32),
                                 idesc, (kb0 + j > 0 || kk > 0) ? 1u : 0u);
                }
              }
            }
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
      }
      umma_commit_pair(drain, 0x1);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 200000000ull) {
      }
    }
  } else {
    // two warps per TMEM lane quarter, one per half of the tile's 32-column chunks
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int m = quarter * 32 + static_cast<int>(lane);
    const uint32_t leader_tempty0 = cluster_addr(smem_u32(&tempty[0]), 0);
    float gn_n = 0.0f, gn_mean = 0.0f, gn_m2 = 0.0f;  // statistics of group `lane`
    int local = 0;
    for (int t = pair; t < s.num_tiles; t += pairs, ++local) {
      const int mt = t % s.tiles_m;
      const int nt = t / s.tiles_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int box = mt * 2 + static_cast<int>(rank);
      if (box < s.boxes)  // warp-uniform
        conv_store_box<BN>(s, e, out, box, nt, tmem_base + ((quarter * 32) << 16) + acc * BN, m,
                           lane, gn_n, gn_mean, gn_m2, half * (BN / 64), (half + 1) * (BN / 64));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty0 + acc * 8);
    }
    if (e.stats != nullptr) {
      // the two warps of a lane quarter merge their statistics (their groups overlap under
      // depth-to-space) into one record per quarter: record (CTA * 4 + quarter)
      float* xch = stats_xch + (quarter * 32 + static_cast<int>(lane)) * 3;
      if (half == 1) {
        xch[0] = gn_n;
        xch[1] = gn_mean;
        xch[2] = gn_m2;
      }
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
      if (half == 0) {
        chan_merge(gn_n, gn_mean, gn_m2, xch[0], xch[1], xch[2]);
        float* rec = e.stats + GN_STATS_RECORDS + (blockIdx.x * 4 + quarter) * 96 + lane * 3;
        rec[0] = gn_n;
        rec[1] = gn_mean;
        rec[2] = gn_m2;
        if (blockIdx.x == 0 && warp == 2 && lane == 0)
          *reinterpret_cast<int*>(e.stats) = static_cast<int>(gridDim.x) * 4;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs have drained; neither CTA's memory is in use any more
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

}  // namespace kino
