// Bandwidth-bound kernels of the video-VAE decode (channels-last activations, bf16).
#pragma once
#include "kino_common.cuh"
#include "kino_ops.cuh"

namespace kino {

// ----------------------------------------------------------------------------- PixelNorm + SiLU
// Stepwise PixelNorm over channels in the activation dtype (kinomlx/kernels/fused_ops.py:460-476:
// square, mean, + eps, sqrt, divide, each rounded to bf16; the mean accumulates in fp32), then
// SiLU with fp32 opmath (fused_ops.py:40-45, blocks.py:165-168). One warp per voxel.
__global__ void pixel_norm_silu_kernel(const __nv_bfloat16* __restrict__ x,
                                       __nv_bfloat16* __restrict__ out, int64_t voxels, int C,
                                       float eps, int apply_silu) {
  griddep_wait();
  griddep_launch();
  const int64_t warp_global = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= voxels) return;
  const __nv_bfloat16* row = x + warp_global * C;
  __nv_bfloat16* orow = out + warp_global * C;
  const int nvec = C >> 3;
  float v[4][8];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      load8(row + c * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += bf16_round(v[i][j] * v[i][j]);
    }
  }
  s = warp_sum(s);
  const float mean = bf16_round(s / static_cast<float>(C));
  const float shifted = bf16_round(mean + eps);
  const float rms = bf16_round(sqrtf(shifted));
  const float rrms = __frcp_rn(rms);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = div_round_bf16(v[i][j], rms, rrms, 4u);
        o[j] = apply_silu ? silu_round_bf16(y) : y;
      }
      store8(orow + c * 8, o);
    }
  }
}

// The same PixelNorm (+ SiLU) for C in {64, 128, ..., 1024}: C/8 threads per voxel (at most 32),
// each holding C/256 (at least one) 16-byte vectors, so every lane of a warp works (two to four
// voxels per warp at C <= 128) and the group's sum of squares is a shuffle over its own lanes.
// Per-element operations as above; only the fp32 summation order of the mean differs.
template <int C>
__global__ void __launch_bounds__(256)
    pixel_norm_silu_vec_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                               int64_t voxels, float eps, int apply_silu) {
  griddep_wait();
  griddep_launch();
  constexpr int T = C / 8 < 32 ? C / 8 : 32;  // threads per voxel
  constexpr int K = C / (8 * T);              // 16-byte vectors per thread
  constexpr int VW = 32 / T;                  // voxels per warp
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t voxel = warp_global * VW + lane / T;
  const int sub = lane % T;
  const bool live = voxel < voxels;
  const __nv_bfloat16* row = x + (live ? voxel : 0) * C;
  float v[K][8];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (live) {
      load8(row + (k * T + sub) * 8, v[k]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[k][j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += bf16_round(v[k][j] * v[k][j]);
  }
#pragma unroll
  for (int o = T / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (!live) return;
  const float mean = bf16_round(s / static_cast<float>(C));
  const float shifted = bf16_round(mean + eps);
  const float rms = bf16_round(sqrtf(shifted));
  const float rrms = __frcp_rn(rms);
  __nv_bfloat16* orow = out + voxel * C;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float y = div_round_bf16(v[k][j], rms, rrms, 4u);
      o[j] = apply_silu ? silu_round_bf16(y) : y;
    }
    store8(orow + (k * T + sub) * 8, o);
  }
}

// ----------------------------------------------------------------------------- GroupNorm
// Affine GroupNorm with fp32 two-pass statistics over each group's channels and all voxels
// (kinomlx/kernels/fused_ops.py:47-139, 375-409), then optionally SiLU. The statistics need a
// grid-wide reduction: every CTA writes its partial sums for the 32 groups into a caller-owned
// workspace, a one-CTA pass turns them into the mean (then the reciprocal std), and the apply
// pass normalises. Workspace layout (floats): partial[parts][32], mean[32], rstd[32].
constexpr int GN_GROUPS = 32;
constexpr int GN_THREADS = 256;

// pass 0: sum(x); pass 1: sum((x - mean)^2). Each thread's eight channel sums are staged in
// shared memory and thread g < 32 adds group g's entries in a fixed order (rows, then
// channels), so the statistics, and every output bit, are the same on every run.
__global__ void __launch_bounds__(GN_THREADS)
    group_norm_partial_kernel(const __nv_bfloat16* __restrict__ x, int64_t voxels, int C,
                              float* __restrict__ ws, int parts, int pass) {
  griddep_wait();
  griddep_launch();
  __shared__ float part[GN_THREADS * 8];
  const int vec_per_row = C >> 3;
  const int rows_per_iter = GN_THREADS / vec_per_row;  // C <= 2048
  const int cv = threadIdx.x % vec_per_row;
  const int r0 = threadIdx.x / vec_per_row;
  const int gs = C / GN_GROUPS;
  const float* mean = ws + static_cast<int64_t>(parts) * GN_GROUPS;
  float m[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) m[j] = pass ? mean[(cv * 8 + j) / gs] : 0.0f;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (r0 < rows_per_iter) {
    const int64_t per = (voxels + parts - 1) / parts;
    const int64_t begin = blockIdx.x * per;
    const int64_t end = begin + per < voxels ? begin + per : voxels;
    for (int64_t v = begin + r0; v < end; v += rows_per_iter) {
      float f[8];
      load8(x + v * C + cv * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = f[j] - m[j];
        acc[j] += pass ? d * d : f[j];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[threadIdx.x * 8 + j] = acc[j];
  __syncthreads();
  if (threadIdx.x < GN_GROUPS) {
    const int g = threadIdx.x;
    float s = 0.0f;
    for (int r = 0; r < rows_per_iter; ++r)
      for (int c = g * gs; c < (g + 1) * gs; ++c) s += part[(r * vec_per_row + (c >> 3)) * 8 + (c & 7)];
    ws[static_cast<int64_t>(blockIdx.x) * GN_GROUPS + g] = s;
  }
}

// One CTA of 32 threads: reduce the partials of group g; pass 0 writes mean, pass 1 rstd.
__global__ void group_norm_finalize_kernel(float* __restrict__ ws, int parts, int64_t count,
                                           float eps, int pass) {
  griddep_wait();
  griddep_launch();
  const int g = threadIdx.x;
  if (g >= GN_GROUPS) return;
  float s = 0.0f;
  for (int p = 0; p < parts; ++p) s += ws[static_cast<int64_t>(p) * GN_GROUPS + g];
  float* mean = ws + static_cast<int64_t>(parts) * GN_GROUPS;
  float* rstd = mean + GN_GROUPS;
  if (pass == 0) {
    mean[g] = s / static_cast<float>(count);
  } else {
    rstd[g] = rsqrtf(s / static_cast<float>(count) + eps);
  }
}

// Statistics from the producing conv's epilogue (see ConvEpi::stats): combine the records of
// each group into mean and rstd. One CTA of GN_MERGE_THREADS per group; each thread loads its
// few records at once (their latencies overlap), then two block reductions with no division
// inside the loops: the group's count and mean from sum(n_i) and sum(n_i * mean_i), then
// m2 = sum(m2_i + n_i * (mean_i - mean)^2), the exact pooled sum of squared deviations about
// the group mean (every term non-negative, so fp32 sums stay accurate).
constexpr int GN_MERGE_THREADS = 256;

__device__ __forceinline__ float gn_block_sum(float v, float* red) {
  v = warp_sum_f(v);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x & 31) < (GN_MERGE_THREADS / 32) ? red[threadIdx.x & 31] : 0.0f;
  t = warp_sum_f(t);
  __syncthreads();  // red is reused by the next reduction
  return t;
}

__global__ void __launch_bounds__(GN_MERGE_THREADS) group_norm_merge_kernel(
    float* __restrict__ stats, float eps) {
  __shared__ float red[GN_MERGE_THREADS / 32];
  griddep_wait();
  griddep_launch();
  const int g = blockIdx.x;
  const int records = *reinterpret_cast<const int*>(stats);
  const float* base = stats + 128 + g * 3;
  constexpr int PER = 4;  // records per thread held in registers (more are read in a loop)
  float rn[PER], rm[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int r = threadIdx.x + GN_MERGE_THREADS * i;
    const bool ok = r < records;
    rn[i] = ok ? base[r * 96] : 0.0f;
    rm[i] = ok ? base[r * 96 + 1] : 0.0f;
  }
  float n = 0.0f, s = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    n += rn[i];
    s = fmaf(rn[i], rm[i], s);
  }
  for (int r = threadIdx.x + GN_MERGE_THREADS * PER; r < records; r += GN_MERGE_THREADS) {
    n += base[r * 96];
    s = fmaf(base[r * 96], base[r * 96 + 1], s);
  }
  n = gn_block_sum(n, red);
  s = gn_block_sum(s, red);
  const float count = n > 0.0f ? n : 1.0f;
  const float mean = s / count;
  float m2 = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int r = threadIdx.x + GN_MERGE_THREADS * i;
    const float d = rm[i] - mean;
    m2 += fmaf(rn[i] * d, d, r < records ? base[r * 96 + 2] : 0.0f);
  }
  for (int r = threadIdx.x + GN_MERGE_THREADS * PER; r < records; r += GN_MERGE_THREADS) {
    const float* rec = base + r * 96;
    const float d = rec[1] - mean;
    m2 += fmaf(rec[0] * d, d, rec[2]);
  }
  m2 = gn_block_sum(m2, red);
  if (threadIdx.x == 0) {
    stats[4 + g] = mean;
    stats[36 + g] = rsqrtf(m2 / count + eps);
  }
}

// y = (x - mean[g]) * rstd[g] * w + b in fp32, rounded to bf16, then SiLU (special-function
// exp2 and reciprocal; the activation's own rounding dominates). Each thread owns one 8-channel
// vector of every voxel it visits, so its weights, biases and group statistics stay in
// registers; threads of a CTA cover C / 8 vectors x (256 / (C / 8)) voxels per step. The pass
// is HBM-bound: each thread keeps KINO_GN_APPLY_UNROLL 16-byte loads in flight (voxels v,
// v + step, ...) so that the bytes in flight per SM cover the memory latency at the occupancy
// the registers allow.
#ifndef KINO_GN_APPLY_UNROLL
#define KINO_GN_APPLY_UNROLL 4
#endif
__device__ __forceinline__ void gn_apply8(const uint4 raw, const float (&m)[8],
                                          const float (&rs)[8], const float (&w)[8],
                                          const float (&b)[8], int apply_silu,
                                          __nv_bfloat16* dst) {
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
  float o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(u[i]);
    const float y0 = (t.x - m[2 * i]) * rs[2 * i] * w[2 * i] + b[2 * i];
    const float y1 = (t.y - m[2 * i + 1]) * rs[2 * i + 1] * w[2 * i + 1] + b[2 * i + 1];
    o[2 * i] = apply_silu ? silu_fast_f32(bf16_round(y0)) : y0;
    o[2 * i + 1] = apply_silu ? silu_fast_f32(bf16_round(y1)) : y1;
  }
  store8(dst, o);
}

__global__ void __launch_bounds__(256)
    group_norm_apply_kernel(const __nv_bfloat16* __restrict__ x,
                            const __nv_bfloat16* __restrict__ weight,
                            const __nv_bfloat16* __restrict__ bias,
                            __nv_bfloat16* __restrict__ out, int64_t voxels, int C,
                            const float* __restrict__ mean, const float* __restrict__ rstd,
                            int apply_silu) {
  griddep_wait();
  griddep_launch();
  const int gs = C / GN_GROUPS;
  const int vecs = C >> 3;
  const int rows = 256 / vecs;
  const int cv = threadIdx.x % vecs;
  const int r0 = threadIdx.x / vecs;
  if (r0 >= rows) return;
  const int c0 = cv * 8;
  float w[8], b[8], m[8], rs[8];
  load8(weight + c0, w);
  load8(bias + c0, b);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    m[j] = mean[(c0 + j) / gs];
    rs[j] = rstd[(c0 + j) / gs];
  }
  const int64_t step = static_cast<int64_t>(gridDim.x) * rows;
  int64_t v = static_cast<int64_t>(blockIdx.x) * rows + r0;
  constexpr int U = KINO_GN_APPLY_UNROLL;
  for (; v + (U - 1) * step < voxels; v += U * step) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      raw[u] = __ldg(reinterpret_cast<const uint4*>(x + (v + u * step) * C + c0));
#pragma unroll
    for (int u = 0; u < U; ++u) gn_apply8(raw[u], m, rs, w, b, apply_silu, out + (v + u * step) * C + c0);
  }
  for (; v < voxels; v += step)
    gn_apply8(__ldg(reinterpret_cast<const uint4*>(x + v * C + c0)), m, rs, w, b, apply_silu,
              out + v * C + c0);
}

// ----------------------------------------------------------------------------- latent -> BFHWC
// x * std[c] + mean[c] in fp32 from a bf16 BCFHW latent, rounded to bf16 channels-last
// (kinomlx/models/ltx2/video_vae/decoder.py:227-233, ops.py:185-188).
__global__ void latent_to_bfhwc_kernel(const __nv_bfloat16* __restrict__ latent,
                                       const float* __restrict__ stdv,
                                       const float* __restrict__ meanv,
                                       __nv_bfloat16* __restrict__ out, int C, int64_t voxels) {
  griddep_wait();
  griddep_launch();
  const int64_t n = voxels * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const int64_t v = i / C;
    const float val = __bfloat162float(latent[static_cast<int64_t>(c) * voxels + v]);
    out[i] = __float2bfloat16_rn(val * stdv[c] + meanv[c]);
  }
}

// ----------------------------------------------------------------------------- tile blend
// One decoded tile (Ft, h, w, 3 * p * p) bf16 from conv_out: unpatchify (packed channel index
// c * p^2 + pw * p + ph, blocks.py:200-230), widen to fp32 and accumulate decoded * mask into the
// fp32 BCFHW canvas at the tile's pixel offset; the first call for a tile position also adds the
// mask to the weight canvas (tiling.py:1310-1330).
__device__ __forceinline__ float tile_value(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float tile_value(float v) { return v; }

// T: the decoded tile's element type (bf16, or fp32 in the fp32 parity mode).
template <typename T>
__global__ void tile_blend_kernel(const T* __restrict__ dec, int Ft, int ht, int wt,
                                  int channels, int patch, float* __restrict__ canvas,
                                  float* __restrict__ wcanvas, int Hout, int Wout, int y0, int x0,
                                  const float* __restrict__ mask_h, const float* __restrict__ mask_w) {
  griddep_wait();
  griddep_launch();
  // one output row (channel, frame, y) per CTA iteration, the row's pixels across the threads:
  // the index arithmetic is per row, in 32 bits, and the canvas accesses are coalesced
  const int Hp = ht * patch, Wp = wt * patch;
  const int nrows = channels * Ft * Hp;
  const int packed = channels * patch * patch;
  for (int rr = blockIdx.x; rr < nrows; rr += gridDim.x) {
    const int yy = rr % Hp;
    const int cf = rr / Hp;
    const int f = cf % Ft;
    const int c = cf / Ft;
    const int h = yy / patch, ph = yy - (yy / patch) * patch;
    const float mh = mask_h[yy];
    const int64_t src_row = (static_cast<int64_t>(f) * ht + h) * wt * packed +
                            static_cast<int64_t>(c) * patch * patch + ph;
    const int64_t dst_row =
        ((static_cast<int64_t>(c) * Ft + f) * Hout + (y0 + yy)) * static_cast<int64_t>(Wout) + x0;
    const bool first_plane = c == 0 && f == 0;
    for (int xx = threadIdx.x; xx < Wp; xx += blockDim.x) {
      const int w = xx / patch, pw = xx - (xx / patch) * patch;
      const float m = mh * mask_w[xx];
      const float val =
          tile_value(dec[src_row + static_cast<int64_t>(w) * packed + pw * patch]) * m;
      canvas[dst_row + xx] += val;
      if (first_plane) wcanvas[static_cast<int64_t>(y0 + yy) * Wout + x0 + xx] += m;
    }
  }
}

// canvas[c, f, y, x] /= max(weights[y, x], 1e-8) (tiling.py:1369)
__global__ void blend_normalize_kernel(float* __restrict__ canvas,
                                       const float* __restrict__ wcanvas, int64_t planes,
                                       int64_t hw) {
  griddep_wait();
  griddep_launch();
  const int64_t n = planes * hw;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    canvas[i] = canvas[i] / fmaxf(wcanvas[i % hw], 1e-8f);
  }
}

}  // namespace kino
