// Bandwidth-bound kernels of the denoise step. Each restates one reference operation with its
// rounding points, reading and writing every element once.
#pragma once
#include "kino_common.cuh"

namespace kino {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; `red` holds one float per warp. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5;
  const int l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (l < nw) ? red[l] : 0.0f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 r;
  r.x = pack_bf16x2(f[0], f[1]);
  r.y = pack_bf16x2(f[2], f[3]);
  r.z = pack_bf16x2(f[4], f[5]);
  r.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = r;
}

// ----------------------------------------------------------------------------- AdaLN
// out = norm(x) * (1 + scale[b]) + shift[b], norm = LayerNorm (no affine) or RMSNorm (no
// affine), statistics in fp32, the normalised row rounded to bf16, then the modulation in bf16
// arithmetic one operation at a time:
//   kinomlx/models/flux2/transformer.py:56-60 (layer_norm, eps 1e-6)
//   kinomlx/models/ltx2/transformer/transformer.py:16-23 (rms_norm)
//   kinomlx/models/ltx2/transformer/model.py:577-592 (output LayerNorm + shift/scale)
constexpr int ADALN_THREADS = 128;
constexpr int ADALN_MAXV = 8;  // dim <= 128 threads * 8 vectors * 8 = 8192

__global__ void __launch_bounds__(ADALN_THREADS)
    adaln_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int64_t bs_x,
                 const __nv_bfloat16* __restrict__ shift, const __nv_bfloat16* __restrict__ scale,
                 int64_t bs_mod, __nv_bfloat16* __restrict__ out, int64_t ld_out, int64_t bs_out,
                 int rows, int dim, int norm_kind, float eps) {
  griddep_wait();
  griddep_launch();
  // norm_kind: 0 RMSNorm, 1 LayerNorm, 2 none (modulation only,
  // kinomlx/models/ltx2/transformer/transformer.py:34-35)
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int b = blockIdx.y;
  const __nv_bfloat16* xr = x + b * bs_x + static_cast<int64_t>(row) * ld_x;
  __nv_bfloat16* orow = out + b * bs_out + static_cast<int64_t>(row) * ld_out;
  const int nvec = dim >> 3;
  float v[ADALN_MAXV][8];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; ++i) {
    const int c = threadIdx.x + i * ADALN_THREADS;
    if (c < nvec) {
      load8(xr + c * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    }
  }
  float mean = 0.0f;
  if (norm_kind == 1) mean = block_sum(s, red) / static_cast<float>(dim);
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; ++i) {
    const int c = threadIdx.x + i * ADALN_THREADS;
    if (c < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mean;
        q += d * d;
      }
    }
  }
  float rstd = 1.0f;
  if (norm_kind != 2) {
    const float var = block_sum(q, red) / static_cast<float>(dim);
    rstd = rsqrtf(var + eps);
  }
  const __nv_bfloat16* sh = shift + b * bs_mod;
  const __nv_bfloat16* sc = scale + b * bs_mod;
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; ++i) {
    const int c = threadIdx.x + i * ADALN_THREADS;
    if (c < nvec) {
      float fs[8], fc[8], o[8];
      load8(sh + c * 8, fs);
      load8(sc + c * 8, fc);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float n = norm_kind == 2 ? v[i][j] : bf16_round((v[i][j] - mean) * rstd);
        const float one_plus = bf16_round(1.0f + fc[j]);
        o[j] = bf16_round(n * one_plus) + fs[j];
      }
      store8(orow + c * 8, o);
    }
  }
}

// Warp-per-row form of the same modulated norm for dim = 256 * VPL, as a streaming kernel: each
// warp walks rows grid-stride (a few CTAs per SM), and every row arrives by cp.async into the
// warp's two shared-memory row slots, the next row's copy in flight while the current one is
// reduced, so the loads of a whole launch are issued up front without holding registers. A lane
// copies and later reads only its own 16-byte chunks (chunk i * 32 + lane), so the per-thread
// cp.async wait is the only synchronisation a row needs. The row is then held in registers as
// packed bf16 (VPL vectors per lane), reduced with shuffles only, and modulated with shift and
// bf16(1 + scale) from shared memory, filled once per CTA. Same rounding points as adaln_kernel.
constexpr int ADALN_WARPS = 8;

__host__ __device__ constexpr int adaln_stream_smem(int vpl) {
  return ADALN_WARPS * 2 * vpl * 32 * 16;  // two row slots per warp
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}

template <int VPL>
__global__ void __launch_bounds__(ADALN_WARPS * 32)
    adaln_warp_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int64_t bs_x,
                      const __nv_bfloat16* __restrict__ shift,
                      const __nv_bfloat16* __restrict__ scale, int64_t bs_mod,
                      __nv_bfloat16* __restrict__ out, int64_t ld_out, int64_t bs_out, int rows,
                      int norm_kind, float eps) {
  constexpr int DIM = VPL * 256;
  __shared__ uint4 s_shift[DIM / 8];
  __shared__ uint4 s_onep[DIM / 8];  // bf16(1 + scale)
  extern __shared__ uint4 s_rows[];  // [warp][slot][VPL * 32]
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint4* slots = s_rows + warp * 2 * VPL * 32;
  const int step = gridDim.x * ADALN_WARPS;
  const __nv_bfloat16* xb = x + b * bs_x;
  auto issue = [&](int row, int slot) {
    const __nv_bfloat16* xr = xb + static_cast<int64_t>(row) * ld_x;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      cp_async16(slots + slot * VPL * 32 + i * 32 + lane, xr + (i * 32 + lane) * 8);
  };
  int row = blockIdx.x * ADALN_WARPS + warp;
  if (row < rows) issue(row, 0);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  const __nv_bfloat16* sh = shift + b * bs_mod;
  const __nv_bfloat16* sc = scale + b * bs_mod;
  for (int c = threadIdx.x; c < DIM / 8; c += ADALN_WARPS * 32) {
    s_shift[c] = *reinterpret_cast<const uint4*>(sh + c * 8);
    float f[8], o[8];
    load8(sc + c * 8, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 1.0f + f[j];
    uint4 w;
    w.x = pack_bf16x2(o[0], o[1]);
    w.y = pack_bf16x2(o[2], o[3]);
    w.z = pack_bf16x2(o[4], o[5]);
    w.w = pack_bf16x2(o[6], o[7]);
    s_onep[c] = w;
  }
  __syncthreads();
  // a bf16 pair as an fp32 pair (exact)
  auto widen = [](uint32_t w) { return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u)); };
  for (int k = 0; row < rows; row += step, ++k) {
    if (row + step < rows) issue(row + step, (k + 1) & 1);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // this row's copies have landed
    const uint4* mine = slots + (k & 1) * VPL * 32;
    uint32_t wv[VPL][4];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint4 r = mine[i * 32 + lane];
      wv[i][0] = r.x;
      wv[i][1] = r.y;
      wv[i][2] = r.z;
      wv[i][3] = r.w;
    }
    __nv_bfloat16* orow = out + b * bs_out + static_cast<int64_t>(row) * ld_out;
    // statistics on fp32 pairs (sm_100 f32x2 arithmetic), reduced over the warp in fp32
    float mean = 0.0f, rstd = 1.0f;
    if (norm_kind != 2) {
      if (norm_kind == 1) {
        uint64_t s2 = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < VPL; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) s2 = f2_add(s2, widen(wv[i][e]));
        const float2 sv = f2_unpack(s2);
        mean = warp_sum(sv.x + sv.y) / static_cast<float>(DIM);
      }
      const uint64_t nm2 = f2_pack(-mean, -mean);
      uint64_t q2 = f2_pack(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < VPL; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint64_t d = f2_add(widen(wv[i][e]), nm2);
          q2 = f2_fma(d, d, q2);
        }
      const float2 qv = f2_unpack(q2);
      rstd = rsqrtf(warp_sum(qv.x + qv.y) / static_cast<float>(DIM) + eps);
    }
    // n = bf16((x - mean) * rstd) on fp32 pairs, then bf16(bf16(n * (1 + scale)) + shift) as
    // two bf16x2 operations, each the single rounding of an exact product or sum
    const uint64_t nm2 = f2_pack(-mean, -mean), rs2 = f2_pack(rstd, rstd);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = i * 32 + lane;
      const uint4 shv = s_shift[c], opv = s_onep[c];
      const uint32_t sw[4] = {shv.x, shv.y, shv.z, shv.w};
      const uint32_t ow[4] = {opv.x, opv.y, opv.z, opv.w};
      uint32_t res[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t nb = wv[i][e];
        if (norm_kind != 2) {
          const float2 nv = f2_unpack(f2_mul(f2_add(widen(wv[i][e]), nm2), rs2));
          nb = pack_bf16x2(nv.x, nv.y);
        }
        const __nv_bfloat162 prod = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&nb),
                                            *reinterpret_cast<const __nv_bfloat162*>(&ow[e]));
        const __nv_bfloat162 sum = __hadd2(prod, *reinterpret_cast<const __nv_bfloat162*>(&sw[e]));
        res[e] = *reinterpret_cast<const uint32_t*>(&sum);
      }
      *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(res[0], res[1], res[2], res[3]);
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// ----------------------------------------------------------------------------- RMSNorm
// Weighted RMSNorm with fp32 reduction, fp32 scale by (weight + offset), one rounding
// (kinomlx/kernels/fused_ops.py:141-193, 412-457); without a weight, the plain fp32 form.
__global__ void __launch_bounds__(ADALN_THREADS)
    rms_norm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                    __nv_bfloat16* __restrict__ out, int dim, float eps, float offset) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * dim;
  __nv_bfloat16* orow = out + row * dim;
  const int nvec = dim >> 3;
  float v[ADALN_MAXV][8];
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; ++i) {
    const int c = threadIdx.x + i * ADALN_THREADS;
    if (c < nvec) {
      load8(xr + c * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) q = fmaf(v[i][j], v[i][j], q);
    }
  }
  const float inv = rsqrtf(block_sum(q, red) / static_cast<float>(dim) + eps);
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; ++i) {
    const int c = threadIdx.x + i * ADALN_THREADS;
    if (c < nvec) {
      float o[8];
      float fw[8];
      if (w != nullptr) {
        load8(w + c * 8, fw);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float r = v[i][j] * inv;
        if (w != nullptr) r *= fw[j] + offset;
        o[j] = r;
      }
      store8(orow + c * 8, o);
    }
  }
}

// RMSNorm of rows no wider than 1024: one warp per row, NCH 16-byte chunks per lane (the
// block-per-row form above leaves most of its threads idle on narrow rows); same fp32 math.
constexpr int RMS_WARP_THREADS = 256;
template <int NCH>
__global__ void __launch_bounds__(RMS_WARP_THREADS)
    rms_norm_warp_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                         __nv_bfloat16* __restrict__ out, int64_t rows, int dim, float eps,
                         float offset) {
  griddep_wait();
  griddep_launch();
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int nvec = dim >> 3;
  const int64_t wpb = RMS_WARP_THREADS / 32;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.x) * wpb) {
    const __nv_bfloat16* xr = x + row * dim;
    float v[NCH][8];
    float q = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = lane + c * 32;
      if (i < nvec) {
        load8(xr + i * 8, v[c]);
#pragma unroll
        for (int j = 0; j < 8; ++j) q = fmaf(v[c][j], v[c][j], q);
      }
    }
    const float inv = rsqrtf(warp_sum(q) / static_cast<float>(dim) + eps);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = lane + c * 32;
      if (i < nvec) {
        float fw[8];
        if (w != nullptr) load8(w + i * 8, fw);
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float r = v[c][j] * inv;
          if (w != nullptr) r *= fw[j] + offset;
          o[j] = r;
        }
        store8(out + row * dim + i * 8, o);
      }
    }
  }
}

// ----------------------------------------------------------------------------- QK norm + RoPE
// In place on token-major projections (batch, tokens, heads * 128) with row stride ld:
//   norm_kind 0: none; 1: RMSNorm per head (weight[128], kinomlx/models/flux2/transformer.py:68-75);
//             2: RMSNorm over the whole heads*128 row (weight[heads*128],
//                kinomlx/models/ltx2/transformer/attention.py:278-279, 330-339).
//   rope_kind 0: none; 1: adjacent pairs, fp32 tables (tokens, 128) with repeated entries
//                (kinomlx/models/flux2/transformer.py:17-29);
//             2: split halves, fp32 tables (table_batch, heads, tokens, 64)
//                (kinomlx/kernels/split_rope.py:35-56);
//             3: split halves within 64-wide heads (two per 128 columns), tables
//                (table_batch, 2 * heads, tokens, 32) (the LTX audio stream and the
//                audio/video cross-attention, kinomlx/models/ltx2/transformer/attention.py:343-346).
// The normalised value is rounded to bf16 before the rotation, as the reference's separate
// norm and rotate operations are. One CTA per token, 8 threads per head, 16 values per thread.
__global__ void qk_norm_rope_kernel(__nv_bfloat16* __restrict__ x, int64_t ld, int64_t bs,
                                    int heads, const __nv_bfloat16* __restrict__ w, int norm_kind,
                                    int rope_kind, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, int table_batched,
                                    int table_tokens, int table_offset, float eps,
                                    __nv_bfloat16* const* __restrict__ dst_ptrs = nullptr,
                                    int heads_per_rank = 0, int64_t dst_ld = 0,
                                    int64_t dst_row0 = 0, int dst_slot = 0) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int b = blockIdx.y;
  const int h = threadIdx.x >> 3;
  const int u = threadIdx.x & 7;
  __nv_bfloat16* row = x + b * bs + static_cast<int64_t>(t) * ld;
  // element indices held by this thread (two runs of 8)
  int e0, e1;
  if (rope_kind == 2) {
    e0 = h * 128 + u * 8;
    e1 = e0 + 64;
  } else if (rope_kind == 3) {
    e0 = h * 128 + (u >> 2) * 64 + (u & 3) * 8;
    e1 = e0 + 32;
  } else {
    e0 = h * 128 + u * 16;
    e1 = e0 + 8;
  }
  float a[8], c[8];
  load8(row + e0, a);
  load8(row + e1, c);
  if (norm_kind != 0) {
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) q = fmaf(a[j], a[j], fmaf(c[j], c[j], q));
    float tot;
    int width;
    if (norm_kind == 1) {
      tot = q;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
      width = 128;
    } else {
      tot = block_sum(q, red);
      width = heads * 128;
    }
    const float inv = rsqrtf(tot / static_cast<float>(width) + eps);
    float wa[8], wc[8];
    const int wo0 = norm_kind == 1 ? (e0 - h * 128) : e0;
    const int wo1 = norm_kind == 1 ? (e1 - h * 128) : e1;
    load8(w + wo0, wa);
    load8(w + wo1, wc);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a[j] = bf16_round(a[j] * inv * wa[j]);
      c[j] = bf16_round(c[j] * inv * wc[j]);
    }
  }
  if (rope_kind == 1) {
    // adjacent pairs (2i, 2i+1): out = x * cos + perp(x) * sin, perp = (-x[2i+1], x[2i])
    const int tt = table_offset + t;
    const float* cr = cos_t + (table_batched ? static_cast<int64_t>(b) * table_tokens : 0) * 128 +
                      static_cast<int64_t>(tt) * 128;
    const float* sr = sin_t + (table_batched ? static_cast<int64_t>(b) * table_tokens : 0) * 128 +
                      static_cast<int64_t>(tt) * 128;
    const int d0 = e0 - h * 128;
    float ra[8], rc[8];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float c0 = cr[d0 + j], c1 = cr[d0 + j + 1], s0 = sr[d0 + j], s1 = sr[d0 + j + 1];
      ra[j] = __fadd_rn(__fmul_rn(a[j], c0), __fmul_rn(-a[j + 1], s0));
      ra[j + 1] = __fadd_rn(__fmul_rn(a[j + 1], c1), __fmul_rn(a[j], s1));
      const float c2 = cr[d0 + 8 + j], c3 = cr[d0 + 9 + j], s2 = sr[d0 + 8 + j],
                  s3 = sr[d0 + 9 + j];
      rc[j] = __fadd_rn(__fmul_rn(c[j], c2), __fmul_rn(-c[j + 1], s2));
      rc[j + 1] = __fadd_rn(__fmul_rn(c[j + 1], c3), __fmul_rn(c[j], s3));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a[j] = ra[j];
      c[j] = rc[j];
    }
  } else if (rope_kind == 2 || rope_kind == 3) {
    // split halves: first = a (i), second = c (i + half), table entry (b|0, head, t, i); with
    // 64-wide heads (kind 3) the 128 columns hold heads 2h and 2h + 1, half 32
    const int tt = table_offset + t;
    const int64_t base =
        rope_kind == 2
            ? ((static_cast<int64_t>(table_batched ? b : 0) * heads + h) * table_tokens + tt) * 64 +
                  u * 8
            : ((static_cast<int64_t>(table_batched ? b : 0) * 2 * heads + 2 * h + (u >> 2)) *
                   table_tokens + tt) * 32 + (u & 3) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float cs = cos_t[base + j];
      const float sn = sin_t[base + j];
      const float first_c = __fmul_rn(a[j], cs);
      const float second_s = __fmul_rn(c[j], sn);
      const float first_s = __fmul_rn(a[j], sn);
      const float second_c = __fmul_rn(c[j], cs);
      a[j] = __fsub_rn(first_c, second_s);
      c[j] = __fadd_rn(first_s, second_c);
    }
  }
  if (dst_ptrs == nullptr) {
    store8(row + e0, a);
    store8(row + e1, c);
  } else {
    // sequence parallel: head h goes to the receive buffer of the rank that owns it
    const int owner = h / heads_per_rank;
    __nv_bfloat16* dst = dst_ptrs[owner] + (dst_row0 + t) * dst_ld +
                         static_cast<int64_t>(dst_slot) * heads_per_rank * 128 +
                         (h - owner * heads_per_rank) * 128 - h * 128;
    store8(dst + e0, a);
    store8(dst + e1, c);
    __threadfence_system();
  }
}

// Standalone split-half RoPE with the reference kernel's contract: value (B, T, H*2*half) in
// bf16, tables (table_batch, H, T, half) fp32, one fp32 rounding per product, then the
// difference or sum, then the cast (kinomlx/kernels/split_rope.py:35-56, 159-163).
__global__ void split_rope_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ cs,
                                  const float* __restrict__ sn, __nv_bfloat16* __restrict__ out,
                                  int batch, int tokens, int heads, int half, int table_batched) {
  griddep_wait();
  griddep_launch();
  const int64_t n = static_cast<int64_t>(batch) * tokens * heads * half;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % half);
    int64_t r = idx / half;
    const int h = static_cast<int>(r % heads);
    r /= heads;
    const int t = static_cast<int>(r % tokens);
    const int b = static_cast<int>(r / tokens);
    const int64_t row = (static_cast<int64_t>(b) * tokens + t) * (heads * 2 * half) +
                        static_cast<int64_t>(h) * 2 * half + i;
    const int64_t entry =
        ((static_cast<int64_t>(table_batched ? b : 0) * heads + h) * tokens + t) * half + i;
    const float c = cs[entry];
    const float s = sn[entry];
    const float first = __bfloat162float(x[row]);
    const float second = __bfloat162float(x[row + half]);
    const float first_c = __fmul_rn(first, c);
    const float second_s = __fmul_rn(second, s);
    const float first_s = __fmul_rn(first, s);
    const float second_c = __fmul_rn(second, c);
    out[row] = __float2bfloat16_rn(__fsub_rn(first_c, second_s));
    out[row + half] = __float2bfloat16_rn(__fadd_rn(first_s, second_c));
  }
}

// split_rope_kernel for half % 4 == 0: four pairs per thread with 8-byte value and 16-byte table
// loads, one (batch, token) row per CTA iteration with 32-bit index math; identical arithmetic.
__global__ void split_rope_vec4_kernel(const __nv_bfloat16* __restrict__ x,
                                       const float* __restrict__ cs, const float* __restrict__ sn,
                                       __nv_bfloat16* __restrict__ out, int batch, int tokens,
                                       int heads, int half, int table_batched) {
  griddep_wait();
  griddep_launch();
  const int groups = half >> 2;  // four-pair groups per head
  const int per_row = heads * groups;
  const int rows = batch * tokens;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int b = r / tokens;
    const int t = r - b * tokens;
    const int64_t xrow = static_cast<int64_t>(r) * heads * 2 * half;
    for (int j = threadIdx.x; j < per_row; j += blockDim.x) {
      const int h = j / groups;
      const int i = (j - h * groups) * 4;
      const int64_t xo = xrow + static_cast<int64_t>(h) * 2 * half + i;
      const int64_t eo =
          ((static_cast<int64_t>(table_batched ? b : 0) * heads + h) * tokens + t) * half + i;
      const float4 c = *reinterpret_cast<const float4*>(cs + eo);
      const float4 sv = *reinterpret_cast<const float4*>(sn + eo);
      const uint2 fa = *reinterpret_cast<const uint2*>(x + xo);
      const uint2 sa = *reinterpret_cast<const uint2*>(x + xo + half);
      const float2 f01 = unpack_bf16x2(fa.x), f23 = unpack_bf16x2(fa.y);
      const float2 s01 = unpack_bf16x2(sa.x), s23 = unpack_bf16x2(sa.y);
      const float first[4] = {f01.x, f01.y, f23.x, f23.y};
      const float second[4] = {s01.x, s01.y, s23.x, s23.y};
      const float cv[4] = {c.x, c.y, c.z, c.w};
      const float svv[4] = {sv.x, sv.y, sv.z, sv.w};
      float o1[4], o2[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        o1[k] = __fsub_rn(__fmul_rn(first[k], cv[k]), __fmul_rn(second[k], svv[k]));
        o2[k] = __fadd_rn(__fmul_rn(first[k], svv[k]), __fmul_rn(second[k], cv[k]));
      }
      uint2 w1, w2;
      w1.x = pack_bf16x2(o1[0], o1[1]);
      w1.y = pack_bf16x2(o1[2], o1[3]);
      w2.x = pack_bf16x2(o2[0], o2[1]);
      w2.y = pack_bf16x2(o2[2], o2[3]);
      *reinterpret_cast<uint2*>(out + xo) = w1;
      *reinterpret_cast<uint2*>(out + xo + half) = w2;
    }
  }
}

// ----------------------------------------------------------------------------- elementwise
enum ElemKind : int {
  ELEM_GELU = 0,       // fused_ops.py:27-35
  ELEM_SILU = 1,       // fused_ops.py:40-45
  ELEM_CFG = 2,        // flux2/sampling.py:272: u + g * (p - u), bf16 ops
  ELEM_EULER_V = 3,    // flux2/sampling.py:109-113: x + bf16(bf16(dt) * v) in fp32
  ELEM_EULER_X0 = 4,   // ltx2 wrappers.py:49-65 + samplers/steps.py:36-70
  ELEM_EULER_D = 5,    // samplers/steps.py:36-70: d + ratio * (x - d) in fp32
  ELEM_EULER_VS = 6,   // samplers/steps.py:8-33: x + bf16(fp32 delta * v)
};

__global__ void elementwise_kernel(int kind, const __nv_bfloat16* __restrict__ a,
                                   const __nv_bfloat16* __restrict__ bsrc,
                                   __nv_bfloat16* __restrict__ out, int64_t n, float s0, float s1) {
  griddep_wait();
  griddep_launch();
  const int64_t nv = n >> 3;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x[8], y[8], o[8];
    load8(a + i * 8, x);
    if (bsrc != nullptr) load8(bsrc + i * 8, y);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      switch (kind) {
        case ELEM_GELU:
          o[j] = gelu_tanh_f32(x[j]);
          break;
        case ELEM_SILU:
          o[j] = silu_f32(x[j]);
          break;
        case ELEM_CFG: {  // a = cond (positive), b = uncond
          const float d = bf16_round(x[j] - y[j]);
          o[j] = y[j] + bf16_round(s0 * d);
          break;
        }
        case ELEM_EULER_V:  // a = sample, b = velocity, s0 = dt
          o[j] = x[j] + bf16_round(bf16_round(s0) * y[j]);
          break;
        case ELEM_EULER_X0: {  // a = sample, b = velocity, s0 = sigma, s1 = sigma_next / sigma
          const float d = bf16_round(__fsub_rn(x[j], __fmul_rn(s0, y[j])));
          o[j] = __fadd_rn(d, __fmul_rn(s1, __fsub_rn(x[j], d)));
          break;
        }
        case ELEM_EULER_D:  // a = sample, b = denoised, s1 = sigma_next / sigma
          o[j] = __fadd_rn(y[j], __fmul_rn(s1, __fsub_rn(x[j], y[j])));
          break;
        case ELEM_EULER_VS:  // a = sample, b = velocity, s0 = sigma_next - sigma (fp32)
          o[j] = __fadd_rn(x[j], bf16_round(__fmul_rn(s0, y[j])));
          break;
        default:
          o[j] = x[j];
      }
    }
    store8(out + i * 8, o);
  }
}

// out[r, c] = bf16(a[r, c] + b[c]) for a (rows, n) and a broadcast row b (n): the per-block
// modulation tables plus the step's timestep projection
// (kinomlx/models/ltx2/transformer/transformer.py:178-186, model.py:585-587).
__global__ void add_rows_kernel(const __nv_bfloat16* __restrict__ a,
                                const __nv_bfloat16* __restrict__ b,
                                __nv_bfloat16* __restrict__ out, int64_t rows, int64_t n) {
  griddep_wait();
  griddep_launch();
  const int64_t nv = (rows * n) >> 3;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = (i * 8) % n;
    float x[8], y[8], o[8];
    load8(a + i * 8, x);
    load8(b + c, y);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = x[j] + y[j];
    store8(out + i * 8, o);
  }
}

// ----------------------------------------------------------------------------- Ulysses packing
// Sequence parallelism (no reference counterpart: the reference runs on one device). Before an
// attention, each rank's token rows (tokens, heads * 128) are cut into `parts` head groups and
// laid out (parts, tokens, heads/parts * 128), so chunk j goes to rank j in one all-to-all and
// arrives as a contiguous token-major block; after the attention the reverse unpack rebuilds the
// rows, optionally multiplying each head by its gate: bf16(bf16(o) * gate[t, head]).
__global__ void heads_pack_kernel(const __nv_bfloat16* __restrict__ src, int64_t ld,
                                  __nv_bfloat16* __restrict__ dst, int tokens, int width,
                                  int parts) {
  griddep_wait();
  griddep_launch();
  const int chunk = width / parts;  // elements per rank per token
  const int64_t nv = (static_cast<int64_t>(tokens) * width) >> 3;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int t = static_cast<int>(e / width);
    const int c = static_cast<int>(e % width);
    const int j = c / chunk, cc = c % chunk;
    *reinterpret_cast<uint4*>(dst + (static_cast<int64_t>(j) * tokens + t) * chunk + cc) =
        *reinterpret_cast<const uint4*>(src + static_cast<int64_t>(t) * ld + c);
  }
}

__global__ void heads_unpack_kernel(const __nv_bfloat16* __restrict__ src,
                                    __nv_bfloat16* __restrict__ dst, int64_t ld, int tokens,
                                    int width, int parts, const __nv_bfloat16* __restrict__ gate,
                                    int64_t ld_gate) {
  griddep_wait();
  griddep_launch();
  const int chunk = width / parts;
  const int64_t nv = (static_cast<int64_t>(tokens) * width) >> 3;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int t = static_cast<int>(e / width);
    const int c = static_cast<int>(e % width);
    const int j = c / chunk, cc = c % chunk;
    const uint4 raw =
        *reinterpret_cast<const uint4*>(src + (static_cast<int64_t>(j) * tokens + t) * chunk + cc);
    if (gate == nullptr) {
      *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(t) * ld + c) = raw;
    } else {
      const float g = __bfloat162float(gate[static_cast<int64_t>(t) * ld_gate + c / 128]);
      float f[8];
      load8(src + (static_cast<int64_t>(j) * tokens + t) * chunk + cc, f);
#pragma unroll
      for (int q = 0; q < 8; ++q) f[q] = f[q] * g;
      store8(dst + static_cast<int64_t>(t) * ld + c, f);
    }
  }
}

// ----------------------------------------------------------------------------- GEMV (M = batch)
// y[b, n] = sum_k act(x[b, k]) * w[n, k] + bias[n]; act = identity or SiLU rounded to bf16
// (kinomlx/models/flux2/transformer.py:223-258 Modulation / TimestepEmbedding,
//  kinomlx/models/ltx2/transformer/timestep.py:31-85). One warp per output column n streams its
// weight row with 16-byte loads; the activations sit in shared memory as fp32.
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_MAXB = 4;

__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
                const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                __nv_bfloat16* __restrict__ y, int64_t ld_y, int batch, int n, int k, int act) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float xs[];  // [batch][k]
  for (int i = threadIdx.x; i < batch * k; i += blockDim.x) {
    const int b = i / k;
    const int kk = i - b * k;
    float v = __bfloat162float(x[b * ld_x + kk]);
    if (act == 1) v = bf16_round(silu_f32(v));
    xs[i] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int col = blockIdx.x * (GEMV_THREADS / 32) + warp;
  if (col >= n) return;
  const __nv_bfloat16* wr = w + static_cast<int64_t>(col) * k;
  float acc[GEMV_MAXB] = {0.f, 0.f, 0.f, 0.f};
  for (int kk = lane * 8; kk < k; kk += 32 * 8) {
    float wf[8];
    load8(wr + kk, wf);
#pragma unroll
    for (int b = 0; b < GEMV_MAXB; ++b) {
      if (b < batch) {
        const float* xb = xs + b * k + kk;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[b] = fmaf(wf[j], xb[j], acc[b]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < GEMV_MAXB; ++b) {
    if (b < batch) {
      float v = warp_sum(acc[b]);
      if (lane == 0) {
        if (bias != nullptr) v += __bfloat162float(bias[col]);  // addmm: bias in the fp32 sum
        y[b * ld_y + col] = __float2bfloat16_rn(v);
      }
    }
  }
}

// ----------------------------------------------------------------------------- timestep features
// [cos(t * f_i), sin(t * f_i)], f_i = exp(-ln(10000) * i / half), fp32, stored as bf16
// (kinomlx/models/flux2/transformer.py:238-241, kinomlx/models/ltx2/transformer/timestep.py:13-28).
__global__ void timestep_embedding_kernel(const float* __restrict__ t, __nv_bfloat16* __restrict__ out,
                                          int batch, int dim) {
  griddep_wait();
  griddep_launch();
  const int half = dim / 2;
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float f = expf(-9.210340371976184f * static_cast<float>(i) / static_cast<float>(half));
    const float ang = t[b] * f;
    out[b * dim + i] = __float2bfloat16_rn(cosf(ang));
    out[b * dim + half + i] = __float2bfloat16_rn(sinf(ang));
  }
}

}  // namespace kino
