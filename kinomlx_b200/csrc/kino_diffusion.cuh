// Device passes of the LTX-2.5 diffusion video decoder around its neighborhood attention
// (kinomlx/models/ltx2/video_vae/diffusion_decoder.py; the reference's own fused passes are in
// kinomlx/models/ltx2/kernels/diffusion_passes.py:298-647):
//
//   na_qkv_prepare_kernel  the qkv projection's rows (bias added, bf16) -> fp16 q, k and v in
//                          the neighborhood attention's (tokens, heads, 64) layout: per-head
//                          RMSNorm with the learned q / k weights, q times head_dim^-1/2
//                          (diffusion_decoder.py:492-517), and the decoder's absolute 3-D RoPE
//                          on adjacent pairs, the head's pairs split into t, h and w sections
//                          (RotaryPosition3D, diffusion_decoder.py:322-397). One warp per
//                          token, one pair per lane, fp32 arithmetic, the rotation from host-made
//                          fp32 cos / sin tables.
//   strided_copy_kernel    an N-D copy (N <= 8) with any source and destination strides, zero
//                          for a broadcast, and a dtype change among bf16, f16 and fp32: the
//                          decoder's linear pixel shuffles (diffusion_decoder.py:928-971),
//                          spatial patchify / unpatchify (:49-91), edge and trailing-frame
//                          padding (:260-308, :1161-1168) and the fp16 <-> bf16 hand-offs
//                          around the attention. Bandwidth-bound: eight consecutive elements of
//                          the innermost dimension per thread where its size allows (16-byte
//                          loads / stores on a unit-stride side), 32-bit index arithmetic when
//                          the element count allows it.
#pragma once
#include <cuda_fp16.h>

#include "kino_common.cuh"

namespace kino {

constexpr int NAP_THREADS = 256;  // 8 warps, one token each at a time

struct NaPrepParams {
  const __nv_bfloat16* qkv;  // (tokens, >= 3 * heads * 64): [q | k | v]
  int64_t ld;
  __half* q;  // (tokens, heads, 64) each, contiguous
  __half* k;
  __half* v;
  const __nv_bfloat16* wq;  // (64,) learned RMSNorm weights
  const __nv_bfloat16* wk;
  // cos_t (gt, pt) | sin_t | cos_h (gh, ph) | sin_h | cos_w (gw, pw) | sin_w, fp32
  const float* tables;
  int64_t tokens;  // batch * gt * gh * gw
  int heads, gt, gh, gw;
  int pt, ph, pw;  // pairs per section, pt + ph + pw = 32
  float q_scale, eps;
};

// One warp per token (32-bit index arithmetic: the host keeps tokens below 2^31): the token's
// volume position and this lane's rotation are found once, then the warp walks q and k head by
// head (lane = pair) and copies the token's v row, 16 bytes per lane.
__global__ void __launch_bounds__(NAP_THREADS) na_qkv_prepare_kernel(const NaPrepParams p) {
  griddep_wait();
  griddep_launch();
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int width = p.heads * 64;
  // this lane's pair: section and index within it (the same for every token)
  int sec, idx;
  if (lane < p.pt) {
    sec = 0;
    idx = lane;
  } else if (lane < p.pt + p.ph) {
    sec = 1;
    idx = lane - p.pt;
  } else {
    sec = 2;
    idx = lane - p.pt - p.ph;
  }
  const float* cos_tab = p.tables;
  int tab_pairs = p.pt;
  int axis_len = p.gt;
  if (sec >= 1) cos_tab += 2 * p.gt * p.pt;
  if (sec == 1) {
    tab_pairs = p.ph;
    axis_len = p.gh;
  }
  if (sec == 2) {
    cos_tab += 2 * p.gh * p.ph;
    tab_pairs = p.pw;
    axis_len = p.gw;
  }
  const float* sin_tab = cos_tab + axis_len * tab_pairs;
  const float2 wq = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p.wq + 2 * lane));
  const float2 wk = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p.wk + 2 * lane));
  const int vol = p.gt * p.gh * p.gw;
  const int tokens = static_cast<int>(p.tokens);
  const int warps = static_cast<int>(gridDim.x) * (NAP_THREADS / 32);
  for (int tok = static_cast<int>(blockIdx.x) * (NAP_THREADS / 32) + (threadIdx.x >> 5);
       tok < tokens; tok += warps) {
    const int in_vol = tok % vol;
    const int pos = sec == 0 ? in_vol / (p.gh * p.gw)
                             : (sec == 1 ? (in_vol / p.gw) % p.gh : in_vol % p.gw);
    const float c = cos_tab[pos * tab_pairs + idx];
    const float s = sin_tab[pos * tab_pairs + idx];
    const __nv_bfloat16* row = p.qkv + static_cast<int64_t>(tok) * p.ld;
    const int64_t orow = static_cast<int64_t>(tok) * width;
    // q heads then k heads, back to back: four (head, q/k) segments at a time, their loads and
    // shuffle reductions interleaved
    const int jobs = 2 * p.heads;
    for (int j0 = 0; j0 < jobs; j0 += 4) {
      float2 x[4];
      float ss[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = min(j0 + u, jobs - 1);
        x[u] = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(row + j * 64 + 2 * lane));
        ss[u] = x[u].x * x[u].x + x[u].y * x[u].y;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < 4; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + u;
        if (j < jobs) {
          const int which = j >= p.heads ? 1 : 0;  // 0: q, 1: k
          const float inv = rsqrtf(ss[u] * (1.0f / 64.0f) + p.eps);
          const float2 wv = which ? wk : wq;
          const float scale = which ? 1.0f : p.q_scale;
          const float e = x[u].x * inv * wv.x * scale;
          const float o = x[u].y * inv * wv.y * scale;
          const __half2 r = __floats2half2_rn(e * c - o * s, e * s + o * c);
          *reinterpret_cast<__half2*>((which ? p.k : p.q) + orow + (j - which * p.heads) * 64 +
                                      2 * lane) = r;
        }
      }
    }
    for (int ch = lane; ch < width / 8; ch += 32) {
      const uint4 raw = *reinterpret_cast<const uint4*>(row + 2 * width + ch * 8);
      const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
      uint32_t h4[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float2 f = unpack_bf16x2(r4[jj]);
        const __half2 hv = __floats2half2_rn(f.x, f.y);
        h4[jj] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      *reinterpret_cast<uint4*>(p.v + orow + ch * 8) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
    }
  }
}

// ------------------------------------------------------------------------- N-D strided copy
constexpr int COPY_MAX_DIMS = 8;
constexpr int COPY_THREADS = 256;
enum CopyType : int { COPY_BF16 = 0, COPY_F16 = 1, COPY_F32 = 2 };

struct CopyParams {
  const void* src;
  void* dst;
  int ndim;
  int src_type, dst_type;
  int64_t total;
  int64_t size[COPY_MAX_DIMS];
  int64_t src_stride[COPY_MAX_DIMS];  // elements
  int64_t dst_stride[COPY_MAX_DIMS];
};

__device__ __forceinline__ float copy_load(const void* base, int type, int64_t i) {
  if (type == COPY_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  if (type == COPY_F16) return __half2float(static_cast<const __half*>(base)[i]);
  return static_cast<const float*>(base)[i];
}

__device__ __forceinline__ void copy_store(void* base, int type, int64_t i, float v) {
  if (type == COPY_BF16)
    static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else if (type == COPY_F16)
    static_cast<__half*>(base)[i] = __float2half_rn(v);
  else
    static_cast<float*>(base)[i] = v;
}

template <int VEC>
__device__ __forceinline__ void copy_load_run(const void* base, int type, int64_t off,
                                              int64_t stride, float (&v)[VEC]) {
  if (VEC == 8 && stride == 1) {
    if (type != COPY_F32) {
      const void* ptr = static_cast<const uint16_t*>(base) + off;
      if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) {
        const uint4 raw = *static_cast<const uint4*>(ptr);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f;
          if (type == COPY_BF16) {
            f = unpack_bf16x2(w[j]);
          } else {
            f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          }
          v[2 * j] = f.x;
          v[2 * j + 1] = f.y;
        }
        return;
      }
    } else {
      const float* ptr = static_cast<const float*>(base) + off;
      if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) {
        const float4 a = reinterpret_cast<const float4*>(ptr)[0];
        const float4 b = reinterpret_cast<const float4*>(ptr)[1];
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
        v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        return;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) v[j] = copy_load(base, type, off + j * stride);
}

template <int VEC>
__device__ __forceinline__ void copy_store_run(void* base, int type, int64_t off, int64_t stride,
                                               const float (&v)[VEC]) {
  if (VEC == 8 && stride == 1) {
    if (type != COPY_F32) {
      void* ptr = static_cast<uint16_t*>(base) + off;
      if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (type == COPY_BF16) {
            w[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
          } else {
            const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            w[j] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        *static_cast<uint4*>(ptr) = make_uint4(w[0], w[1], w[2], w[3]);
        return;
      }
    } else {
      float* ptr = static_cast<float*>(base) + off;
      if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) {
        reinterpret_cast<float4*>(ptr)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(ptr)[1] = make_float4(v[4], v[5], v[6], v[7]);
        return;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) copy_store(base, type, off + j * stride, v[j]);
}

// Idx: uint32_t when every size and the element count fit 32 bits, else uint64_t. Dimension
// ndim - 1 is the fastest-varying one of the element order; each thread moves VEC consecutive
// elements of it (VEC divides its size).
template <typename Idx, int VEC>
__global__ void __launch_bounds__(COPY_THREADS) strided_copy_kernel(const CopyParams p) {
  griddep_wait();
  griddep_launch();
  const int last = p.ndim - 1;
  Idx size[COPY_MAX_DIMS];
#pragma unroll
  for (int d = 0; d < COPY_MAX_DIMS; ++d) size[d] = static_cast<Idx>(p.size[d]);
  const Idx inner = static_cast<Idx>(p.size[last] / VEC);
  const int64_t s_last = p.src_stride[last], d_last = p.dst_stride[last];
  const Idx runs = static_cast<Idx>(p.total / VEC);
  for (Idx e = static_cast<Idx>(blockIdx.x) * COPY_THREADS + threadIdx.x; e < runs;
       e += static_cast<Idx>(gridDim.x) * COPY_THREADS) {
    Idx rest = e / inner;
    const int64_t c_last = static_cast<int64_t>(e - rest * inner) * VEC;
    int64_t so = c_last * s_last, dof = c_last * d_last;
#pragma unroll
    for (int d = COPY_MAX_DIMS - 2; d >= 0; --d) {
      if (d < last) {
        const Idx q = rest / size[d];
        const Idx c = rest - q * size[d];
        rest = q;
        so += static_cast<int64_t>(c) * p.src_stride[d];
        dof += static_cast<int64_t>(c) * p.dst_stride[d];
      }
    }
    float v[VEC];
    copy_load_run<VEC>(p.src, p.src_type, so, s_last, v);
    copy_store_run<VEC>(p.dst, p.dst_type, dof, d_last, v);
  }
}

}  // namespace kino
