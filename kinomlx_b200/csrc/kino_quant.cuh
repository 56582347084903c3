// Dequantisation of group-quantised linear weights into bf16 for the tcgen05 GEMM.
//
// Restates the weight formats the reference's packed linears consume through MLX's
// quantized_matmul (kinomlx/models/ltx2/weights/quantization.py:17-43, modes and default group
// sizes kinomlx/models/ltx2/weights/tensors.py:185-203):
//   affine  w = scale * q + bias, q unsigned (2, 4 or 8 bits), scale and bias bf16 per group;
//   mxfp8   E4M3 element x E8M0 scale 2^(e - 127) per group of 32 (OCP Microscaling v1.0);
//   mxfp4   E2M1 element x E8M0 scale per group of 32;
//   nvfp4   E2M1 element x E4M3 scale per group of 16.
// Codes are packed along a row, little-endian inside uint32 words. The float modes dequantise
// exactly in fp32 (a short-mantissa element times a power of two or an E4M3 scale); affine is one
// fp32 fma. Each result is rounded to bf16 once.
//
// One CTA per 64 x 64 tile (the last one narrower when cols is not a multiple of 64): every
// thread decodes 16 consecutive codes of one row (one group scale: groups are multiples of 16)
// into a shared-memory tile, which is then written either in the packed orientation or
// transposed (the reference's pretransposed weights are packed from weight.T, i.e. along the
// output dimension; the GEMM wants (out, in) rows).
#pragma once
#include "kino_common.cuh"

namespace kino {

constexpr int DQ_TILE = 64;
constexpr int DQ_THREADS = 256;

__device__ __forceinline__ float dq_e4m3(uint32_t c) {
  const uint32_t e = (c >> 3) & 0xFu, m = c & 0x7u;
  float v;
  if ((c & 0x7Fu) == 0x7Fu) {
    v = __uint_as_float(0x7FC00000u);
  } else if (e == 0) {
    v = static_cast<float>(m) * 0.001953125f;  // m / 8 * 2^-6
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));  // (1 + m/8) * 2^(e - 7)
  }
  return (c & 0x80u) ? -v : v;
}

__device__ __forceinline__ float dq_e2m1(uint32_t c) {
  const uint32_t e = (c >> 1) & 0x3u, m = c & 0x1u;
  const float v = e == 0 ? 0.5f * static_cast<float>(m)
                         : __uint_as_float(((e + 126u) << 23) | (m << 22));  // (1 + m/2) 2^(e-1)
  return (c & 0x8u) ? -v : v;
}

__device__ __forceinline__ float dq_e8m0(uint32_t c) {
  c &= 0xFFu;
  if (c == 255u) return __uint_as_float(0x7FC00000u);
  if (c == 0u) return __uint_as_float(0x00400000u);  // 2^-127 (an fp32 subnormal)
  return __uint_as_float(c << 23);
}

// out = dequantised (rows, cols) codes, or its transpose (cols, rows) when transpose_out.
// mode: 0 affine, 1 mxfp8, 2 mxfp4, 3 nvfp4.
template <int BITS>
__global__ void __launch_bounds__(DQ_THREADS)
    dequant_kernel(const uint32_t* __restrict__ words, const void* __restrict__ scales,
                   const __nv_bfloat16* __restrict__ biases, __nv_bfloat16* __restrict__ out,
                   int64_t rows, int64_t cols, int mode, int group, int transpose_out) {
  griddep_wait();
  griddep_launch();
  __shared__ __align__(16) __nv_bfloat16 tile[DQ_TILE][DQ_TILE + 8];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * DQ_TILE;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * DQ_TILE;
  const int tr = threadIdx.x >> 2;        // tile row
  const int tc = (threadIdx.x & 3) * 16;  // first of the thread's 16 columns
  const int64_t r = r0 + tr;
  const bool live_cols = c0 + tc < cols;  // cols is a multiple of 16: whole segments only
  if (r < rows && live_cols) {
    constexpr int PER = 32 / BITS;  // codes per word
    const int64_t words_per_row = cols / PER;
    const uint32_t* wp = words + r * words_per_row + (c0 + tc) / PER;
    const int64_t gidx = r * (cols / group) + (c0 + tc) / group;
    float sc = 1.0f, bs = 0.0f;
    if (mode == 0) {
      sc = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(scales)[gidx]);
      bs = __bfloat162float(biases[gidx]);
    } else {
      const uint32_t code = reinterpret_cast<const uint8_t*>(scales)[gidx];
      sc = mode == 3 ? dq_e4m3(code) : dq_e8m0(code);
    }
#pragma unroll
    for (int wi = 0; wi < 16 / PER; ++wi) {
      const uint32_t word = __ldg(wp + wi);
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const uint32_t q = (word >> (k * BITS)) & ((1u << BITS) - 1u);
        float v;
        if (mode == 0)
          v = fmaf(sc, static_cast<float>(q), bs);
        else
          v = (mode == 1 ? dq_e4m3(q) : dq_e2m1(q)) * sc;
        tile[tr][tc + wi * PER + k] = __float2bfloat16_rn(v);
      }
    }
  }
  __syncthreads();
  if (!transpose_out) {
    if (r < rows && live_cols) {
      const uint4* src = reinterpret_cast<const uint4*>(&tile[tr][tc]);
      uint4* dst = reinterpret_cast<uint4*>(out + r * cols + c0 + tc);
      dst[0] = src[0];
      dst[1] = src[1];
    }
  } else {
    // thread (column tr of the tile, rows tc .. tc + 15): out[c0 + tr][r0 + tc ...]
    const int64_t oc = c0 + tr;
    if (oc >= cols) return;
    __align__(16) __nv_bfloat16 v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = tile[tc + i][tr];
    __nv_bfloat16* dst = out + oc * rows + r0 + tc;
    if (r0 + tc + 16 <= rows) {
      reinterpret_cast<uint4*>(dst)[0] = reinterpret_cast<const uint4*>(v)[0];
      reinterpret_cast<uint4*>(dst)[1] = reinterpret_cast<const uint4*>(v)[1];
    } else {
      for (int i = 0; i < 16 && r0 + tc + i < rows; ++i) dst[i] = v[i];
    }
  }
}

// Two E4M3 codes (the low byte first) to two f16 values: exact, E4M3 being a subset of f16.
__device__ __forceinline__ float2 dq_e4m3x2(uint32_t two_codes) {
  uint32_t h;
  const uint16_t a = static_cast<uint16_t>(two_codes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(a));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

constexpr int DQ8_THREADS = 256;

// mxfp8 in the packed orientation (codes along each output row, the GEMM's K): the matrix as
// one flat sequence of 8-code chunks (the rows are contiguous, groups of 32 never straddle
// them); lane l of a warp takes chunk l of each 32-chunk run, so every load (8 bytes of codes)
// and store (16 bytes of bf16) instruction of the warp is one contiguous segment. Four chunks
// per thread are in flight at a time, grid-stride. Codes go through the hardware E4M3 -> f16
// conversion (exact), then the same fp32 product with the group's power-of-two scale and the
// single bf16 rounding as dequant_kernel.
__device__ __forceinline__ uint4 dq8_chunk(uint2 c, float sc) {
  const float2 a = dq_e4m3x2(c.x & 0xFFFFu), b = dq_e4m3x2(c.x >> 16);
  const float2 d = dq_e4m3x2(c.y & 0xFFFFu), e = dq_e4m3x2(c.y >> 16);
  return make_uint4(pack_bf16x2(a.x * sc, a.y * sc), pack_bf16x2(b.x * sc, b.y * sc),
                    pack_bf16x2(d.x * sc, d.y * sc), pack_bf16x2(e.x * sc, e.y * sc));
}

__global__ void __launch_bounds__(DQ8_THREADS)
    dequant_mxfp8_rows_kernel(const uint2* __restrict__ codes, const uint8_t* __restrict__ scales,
                              uint4* __restrict__ out, int64_t chunks) {
  griddep_wait();
  griddep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * DQ8_THREADS;
  int64_t e = static_cast<int64_t>(blockIdx.x) * DQ8_THREADS + threadIdx.x;
  for (; e + 3 * stride < chunks; e += 4 * stride) {
    uint2 c[4];
    float sc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      c[u] = __ldg(codes + e + u * stride);
      sc[u] = dq_e8m0(__ldg(scales + (e + u * stride) / 4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) out[e + u * stride] = dq8_chunk(c[u], sc[u]);
  }
  for (; e < chunks; e += stride) out[e] = dq8_chunk(__ldg(codes + e), dq_e8m0(__ldg(scales + e / 4)));
}

// mxfp8 packed from weight.T (the reference's pretransposed weights: codes along the output
// dimension, `rows` = input features) into the GEMM's (out, in) bf16 rows, without a shared-
// memory pass: a warp takes 64 code rows x 32 code columns; lane l decodes its two rows' 32-code
// groups (full 32-byte sectors) and writes, for each of the 32 columns, the bf16 pair of its two
// rows, so each store instruction of the warp fills one contiguous 128-byte output segment.
__global__ void __launch_bounds__(DQ8_THREADS)
    dequant_mxfp8_cols_kernel(const uint4* __restrict__ codes, const uint8_t* __restrict__ scales,
                              uint32_t* __restrict__ out, int64_t rows, int64_t cols) {
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t col_tasks = cols / 32;
  const int64_t tasks = (rows + 63) / 64 * col_tasks;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (DQ8_THREADS / 32);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (DQ8_THREADS / 32) + (threadIdx.x >> 5);
       t < tasks; t += warps) {
    const int64_t c0 = (t % col_tasks) * 32;
    const int64_t r = (t / col_tasks) * 64 + 2 * lane;  // rows r, r + 1 (rows is even)
    if (r >= rows) continue;
    const int64_t g0 = r * col_tasks + c0 / 32, g1 = g0 + col_tasks;
    const uint4 a0 = __ldg(codes + 2 * g0), b0 = __ldg(codes + 2 * g0 + 1);
    const uint4 a1 = __ldg(codes + 2 * g1), b1 = __ldg(codes + 2 * g1 + 1);
    const float s0 = dq_e8m0(__ldg(scales + g0)), s1 = dq_e8m0(__ldg(scales + g1));
    const uint32_t w0[8] = {a0.x, a0.y, a0.z, a0.w, b0.x, b0.y, b0.z, b0.w};
    const uint32_t w1[8] = {a1.x, a1.y, a1.z, a1.w, b1.x, b1.y, b1.z, b1.w};
    uint32_t* dst = out + (c0 * rows + r) / 2;  // out[c0][r .. r + 1] as one bf16 pair
    const int64_t col_stride = rows / 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 x = dq_e4m3x2((w0[i] >> (16 * h)) & 0xFFFFu);
        const float2 y = dq_e4m3x2((w1[i] >> (16 * h)) & 0xFFFFu);
        const int j = 4 * i + 2 * h;
        dst[j * col_stride] = pack_bf16x2(x.x * s0, y.x * s1);
        dst[(j + 1) * col_stride] = pack_bf16x2(x.y * s0, y.y * s1);
      }
    }
  }
}

}  // namespace kino
