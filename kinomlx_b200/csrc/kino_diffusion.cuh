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
//                          (token, head) of q or k, one pair per lane, fp32 arithmetic, the
//                          rotation from host-made fp32 cos / sin tables.
//   strided_copy_kernel    an N-D copy (N <= 8) with any source and destination strides, zero
//                          for a broadcast, and a dtype change among bf16, f16 and fp32: the
//                          decoder's linear pixel shuffles (diffusion_decoder.py:928-971),
//                          spatial patchify / unpatchify (:49-91), edge and trailing-frame
//                          padding (:260-308, :1161-1168) and the fp16 <-> bf16 hand-offs
//                          around the attention. Bandwidth-bound; one element per thread with
//                          32-bit index arithmetic when the element count allows it.
#pragma once
#include <cuda_fp16.h>

#include "kino_common.cuh"

namespace kino {

constexpr int NAP_THREADS = 256;  // 8 warps, each on (token, head) jobs of q then k

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

__global__ void __launch_bounds__(NAP_THREADS) na_qkv_prepare_kernel(const NaPrepParams p) {
  griddep_wait();
  griddep_launch();
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (NAP_THREADS / 32);
  const int64_t jobs = p.tokens * p.heads * 2;
  const int width = p.heads * 64;
  // this lane's pair: section and index within it (the same for every job)
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
  if (sec >= 1) cos_tab += 2 * static_cast<int64_t>(p.gt) * p.pt;
  if (sec == 1) tab_pairs = p.ph;
  if (sec == 2) {
    cos_tab += 2 * static_cast<int64_t>(p.gh) * p.ph;
    tab_pairs = p.pw;
  }
  const int64_t axis_len = sec == 0 ? p.gt : (sec == 1 ? p.gh : p.gw);
  const float* sin_tab = cos_tab + axis_len * tab_pairs;
  for (int64_t job = static_cast<int64_t>(blockIdx.x) * (NAP_THREADS / 32) + (threadIdx.x >> 5);
       job < jobs; job += warps) {
    const int which = static_cast<int>(job & 1);  // 0: q, 1: k
    const int64_t th = job >> 1;
    const int head = static_cast<int>(th % p.heads);
    const int64_t tok = th / p.heads;
    const int64_t in_vol = tok % (static_cast<int64_t>(p.gt) * p.gh * p.gw);
    const int w = static_cast<int>(in_vol % p.gw);
    const int h = static_cast<int>((in_vol / p.gw) % p.gh);
    const int t = static_cast<int>(in_vol / (static_cast<int64_t>(p.gw) * p.gh));
    const __nv_bfloat16* src = p.qkv + tok * p.ld + which * width + head * 64 + 2 * lane;
    const float2 x = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src));
    float ss = x.x * x.x + x.y * x.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss * (1.0f / 64.0f) + p.eps);
    const float2 wv =
        unpack_bf16x2(*reinterpret_cast<const uint32_t*>((which ? p.wk : p.wq) + 2 * lane));
    float e = x.x * inv * wv.x;
    float o = x.y * inv * wv.y;
    if (which == 0) {
      e *= p.q_scale;
      o *= p.q_scale;
    }
    const int pos = sec == 0 ? t : (sec == 1 ? h : w);
    const float c = cos_tab[static_cast<int64_t>(pos) * tab_pairs + idx];
    const float s = sin_tab[static_cast<int64_t>(pos) * tab_pairs + idx];
    const __half2 r = __floats2half2_rn(e * c - o * s, e * s + o * c);
    __half* dst = (which ? p.k : p.q) + tok * width + head * 64 + 2 * lane;
    *reinterpret_cast<__half2*>(dst) = r;
  }
  // v: 8 columns per thread
  const int64_t vchunks = p.tokens * (width / 8);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * NAP_THREADS + threadIdx.x; i < vchunks;
       i += static_cast<int64_t>(gridDim.x) * NAP_THREADS) {
    const int64_t tok = i / (width / 8);
    const int col = static_cast<int>(i % (width / 8)) * 8;
    const uint4 raw = *reinterpret_cast<const uint4*>(p.qkv + tok * p.ld + 2 * width + col);
    const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t h4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(r4[j]);
      const __half2 hv = __floats2half2_rn(f.x, f.y);
      h4[j] = *reinterpret_cast<const uint32_t*>(&hv);
    }
    *reinterpret_cast<uint4*>(p.v + tok * width + col) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
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

// Idx: uint32_t when every size and the element count fit 32 bits, else uint64_t. Dimension
// ndim - 1 is the fastest-varying one of the element order.
template <typename Idx>
__global__ void __launch_bounds__(COPY_THREADS) strided_copy_kernel(const CopyParams p) {
  griddep_wait();
  griddep_launch();
  Idx size[COPY_MAX_DIMS];
#pragma unroll
  for (int d = 0; d < COPY_MAX_DIMS; ++d) size[d] = static_cast<Idx>(p.size[d]);
  for (Idx e = static_cast<Idx>(blockIdx.x) * COPY_THREADS + threadIdx.x;
       e < static_cast<Idx>(p.total); e += static_cast<Idx>(gridDim.x) * COPY_THREADS) {
    Idx rest = e;
    int64_t so = 0, dof = 0;
#pragma unroll
    for (int d = COPY_MAX_DIMS - 1; d >= 0; --d) {
      if (d < p.ndim) {
        const Idx c = rest % size[d];
        rest /= size[d];
        so += static_cast<int64_t>(c) * p.src_stride[d];
        dof += static_cast<int64_t>(c) * p.dst_stride[d];
      }
    }
    copy_store(p.dst, p.dst_type, dof, copy_load(p.src, p.src_type, so));
  }
}

}  // namespace kino
