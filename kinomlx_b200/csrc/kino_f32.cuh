// fp32 parity mode: the Flux2 block operators in single precision on the CUDA cores.
//
// The tensor cores have no fp32 MMA (kind::tf32 keeps 10 mantissa bits), and BASELINE's fp32 gate
// (per-op max relative error <= 1e-4 against the reference's fp32 graph) needs full fp32
// products. These kernels are the fp32 twins of the bf16 path's operators: every product and
// sum in fp32 with the reference's operation order (separate roundings where the reference's
// graph has separate operations, so no fused multiply-add in the epilogues), nothing rounded to
// a narrower type. They are correctness kernels first; the GEMM still uses the usual SIMT
// blocking (128 x 128 tiles, 8 x 8 outputs per thread, double-buffered shared memory).
#pragma once

#include <cuda_runtime.h>
#include <math_constants.h>

#include "kino_common.cuh"

namespace kino {

// ---------------------------------------------------------------- GEMM
constexpr int F32_BM = 128;
constexpr int F32_BN = 128;
constexpr int F32_BK = 16;
constexpr int F32_PAD = 4;  // keeps float4 alignment, halves the transposed-store conflicts
constexpr int F32_THREADS = 256;

struct F32Epi {
  // EPI_NONE (0), EPI_GELU (1), EPI_GATED_RESIDUAL (2), EPI_EULER (3), EPI_SIGMOID2 (4),
  // EPI_EULER_X0 (5)
  int kind;
  const float* bias;
  const float* residual;
  int64_t ld_res, bs_res;
  const float* gate;
  int64_t bs_gate;
  int64_t act_col_begin;
  float scalar;
  const float* aux;
  int64_t ld_aux, bs_aux;
  float scalar2;
};

// tanh-GELU exactly as the reference formula reads in fp32: the inner argument clamped to +-10
// and the library tanh (kinomlx/kernels/fused_ops.py:27-35).
__device__ __forceinline__ float gelu_tanh_exact_f32(float x) {
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, cube));
  const float t = tanhf(fminf(fmaxf(inner, -10.0f), 10.0f));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// x / (1 + exp(-x)) with the library exp and an IEEE divide (kinomlx/kernels/fused_ops.py:40-45).
__device__ __forceinline__ float silu_exact_f32(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

// out[b, i, j] = epilogue(sum_k x[b, i, k] * w[j, k]). Grid (ceil(n/128), ceil(m/128), batch).
// k % 4 == 0 and 16-byte aligned rows (checked by the host). `out` may alias `residual` or `aux`
// (each element is read by the thread that writes it), never `x` or `w`.
__global__ void __launch_bounds__(F32_THREADS, 2)
    gemm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w, float* out, int m,
                    int n, int k, int64_t ldx, int64_t bsx, int64_t ldw, int64_t ldo, int64_t bso,
                    F32Epi e) {
  __shared__ __align__(16) float As[2][F32_BK][F32_BM + F32_PAD];
  __shared__ __align__(16) float Ws[2][F32_BK][F32_BN + F32_PAD];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int b = blockIdx.z;
  const int row0 = blockIdx.y * F32_BM;
  const int col0 = blockIdx.x * F32_BN;
  const float* xb = x + static_cast<int64_t>(b) * bsx;

  // loader: each thread moves rows lr and lr + 64 of the A and W tiles, four k values each
  const int lr = tid >> 2;
  const int lk = (tid & 3) * 4;
  float4 ra[2], rw[2];
  auto load = [&](int k0) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int kk = k0 + lk;
      const int r = row0 + lr + 64 * p;
      const int c = col0 + lr + 64 * p;
      ra[p] = (r < m && kk < k) ? *reinterpret_cast<const float4*>(xb + static_cast<int64_t>(r) * ldx + kk)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      rw[p] = (c < n && kk < k) ? *reinterpret_cast<const float4*>(w + static_cast<int64_t>(c) * ldw + kk)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int r = lr + 64 * p;
      As[buf][lk + 0][r] = ra[p].x;
      As[buf][lk + 1][r] = ra[p].y;
      As[buf][lk + 2][r] = ra[p].z;
      As[buf][lk + 3][r] = ra[p].w;
      Ws[buf][lk + 0][r] = rw[p].x;
      Ws[buf][lk + 1][r] = rw[p].y;
      Ws[buf][lk + 2][r] = rw[p].z;
      Ws[buf][lk + 3][r] = rw[p].w;
    }
  };

  // compute: thread (ty, tx) owns rows {ty*4 + i, 64 + ty*4 + i} x cols {tx*4 + j, 64 + tx*4 + j}
  const int ty = tid >> 4;
  const int tx = tid & 15;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int ktiles = (k + F32_BK - 1) / F32_BK;
  load(0);
  store(0);
  __syncthreads();
  for (int t = 0; t < ktiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ktiles) load((t + 1) * F32_BK);
#pragma unroll
    for (int kk = 0; kk < F32_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Ws[buf][kk][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
    }
    if (t + 1 < ktiles) store(buf ^ 1);
    __syncthreads();
  }

  float* ob = out + static_cast<int64_t>(b) * bso;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (c >= n) continue;
      float v = acc[i][j];
      if (e.bias != nullptr) v = __fadd_rn(v, e.bias[c]);
      if (e.kind == 1) {
        if (c >= e.act_col_begin) v = gelu_tanh_exact_f32(v);
      } else if (e.kind == 2) {
        const float res = e.residual[static_cast<int64_t>(b) * e.bs_res + static_cast<int64_t>(r) * e.ld_res + c];
        v = __fadd_rn(res, __fmul_rn(e.gate[static_cast<int64_t>(b) * e.bs_gate + c], v));
      } else if (e.kind == 3) {
        const float cur = e.aux[static_cast<int64_t>(b) * e.bs_aux + static_cast<int64_t>(r) * e.ld_aux + c];
        v = __fadd_rn(cur, __fmul_rn(e.scalar, v));
      } else if (e.kind == 4) {
        // 2 * sigmoid(v) (kinomlx/models/ltx2/transformer/attention.py:298-303)
        v = __fmul_rn(2.0f, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))));
      } else if (e.kind == 5) {
        // x0 = x - sigma * v, then x0 + ratio * (x - x0) (ltx2/transformer/wrappers.py:49-65,
        // samplers/steps.py:36-70)
        const float cur = e.aux[static_cast<int64_t>(b) * e.bs_aux + static_cast<int64_t>(r) * e.ld_aux + c];
        const float x0 = __fsub_rn(cur, __fmul_rn(e.scalar, v));
        v = __fadd_rn(x0, __fmul_rn(e.scalar2, __fsub_rn(cur, x0)));
      }
      ob[static_cast<int64_t>(r) * ldo + c] = v;
    }
  }
}

// ---------------------------------------------------------------- attention
// softmax(q k^T * scale) v per (batch, head) with head_dim 128, token-major operands, online
// softmax over 64-key blocks (running maximum and sum in fp32, library exp). A CTA holds 64
// queries of one head; grid (ceil(tq/64), heads, batch). `out` may alias `q` (a CTA reads its
// own query rows once, before it writes them, and no other CTA reads them).
constexpr int FA32_BQ = 64;
constexpr int FA32_BK = 64;
constexpr int FA32_D = 128;
constexpr int FA32_PS = 72;  // P row stride: the softmax pass reads and writes it conflict-free
constexpr int FA32_THREADS = 256;

struct Fa32Smem {
  float qt[FA32_D][FA32_BQ];     // Q transposed (head-dim-major)
  float kt[FA32_D][FA32_BK];     // K block transposed
  float v[FA32_BK][FA32_D];      // V block
  float pt[FA32_BK][FA32_PS];    // scores, then probabilities, key-major
  float alpha[FA32_BQ];          // per-row rescale of the running output
  float lsum[FA32_BQ];           // final row sums
};

__global__ void __launch_bounds__(FA32_THREADS, 1)
    attention_f32_kernel(const float* q, const float* __restrict__ k,
                         const float* __restrict__ vv, float* out, int tq, int tk, int64_t ld_q,
                         int64_t bs_q, int64_t ld_k, int64_t bs_k, int64_t ld_v, int64_t bs_v,
                         int64_t ld_o, int64_t bs_o, float scale, const float* __restrict__ gate,
                         int64_t ld_g, int64_t bs_g, const float* __restrict__ key_bias,
                         int64_t ld_bias) {
  extern __shared__ __align__(16) unsigned char fa32_raw[];
  Fa32Smem& s = *reinterpret_cast<Fa32Smem*>(fa32_raw);
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = blockIdx.x * FA32_BQ;
  const float* qb = q + static_cast<int64_t>(b) * bs_q + h * FA32_D;
  const float* kb = k + static_cast<int64_t>(b) * bs_k + h * FA32_D;
  const float* vb = vv + static_cast<int64_t>(b) * bs_v + h * FA32_D;

  // Q tile, transposed: consecutive lanes take consecutive tokens (conflict-free stores)
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int idx = it * FA32_THREADS + tid;
    const int row = idx & 63;
    const int c4 = idx >> 6;
    const int t = q0 + row;
    const float4 x = t < tq ? *reinterpret_cast<const float4*>(qb + static_cast<int64_t>(t) * ld_q + c4 * 4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    s.qt[c4 * 4 + 0][row] = x.x;
    s.qt[c4 * 4 + 1][row] = x.y;
    s.qt[c4 * 4 + 2][row] = x.z;
    s.qt[c4 * 4 + 3][row] = x.w;
  }

  // S / P mapping: thread (ty, tx) owns rows ty*4 + i, keys tx*4 + j
  const int ty = tid >> 4;
  const int tx = tid & 15;
  // softmax mapping: four threads of one warp per row, keys interleaved by 4
  const int sr = (tid >> 5) * 8 + (tid & 7);
  const int sq = (tid & 31) >> 3;
  float m_run = -CUDART_INF_F;
  float l_run = 0.f;
  float o[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 8; ++c) o[i][c] = 0.f;

  const int kblocks = (tk + FA32_BK - 1) / FA32_BK;
  for (int kbk = 0; kbk < kblocks; ++kbk) {
    const int k0 = kbk * FA32_BK;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int idx = it * FA32_THREADS + tid;
      {  // K transposed
        const int row = idx & 63;
        const int c4 = idx >> 6;
        const int t = k0 + row;
        const float4 x = t < tk ? *reinterpret_cast<const float4*>(kb + static_cast<int64_t>(t) * ld_k + c4 * 4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        s.kt[c4 * 4 + 0][row] = x.x;
        s.kt[c4 * 4 + 1][row] = x.y;
        s.kt[c4 * 4 + 2][row] = x.z;
        s.kt[c4 * 4 + 3][row] = x.w;
      }
      {  // V row-major
        const int row = idx >> 5;
        const int c4 = idx & 31;
        const int t = k0 + row;
        const float4 x = t < tk ? *reinterpret_cast<const float4*>(vb + static_cast<int64_t>(t) * ld_v + c4 * 4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(&s.v[row][c4 * 4]) = x;
      }
    }
    __syncthreads();

    // S = (Q K^T) * scale for this thread's 4 x 4 block; keys past tk are -inf
    float sacc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sacc[i][j] = 0.f;
#pragma unroll 8
    for (int d = 0; d < FA32_D; ++d) {
      const float4 a = *reinterpret_cast<const float4*>(&s.qt[d][ty * 4]);
      const float4 c = *reinterpret_cast<const float4*>(&s.kt[d][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sacc[i][j] = fmaf(av[i], cv[j], sacc[i][j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = k0 + tx * 4 + j;
      const bool valid = key < tk;
      // an additive key bias (a text mask) joins the scaled score, as the reference adds it
      const float bias = (valid && key_bias != nullptr)
                             ? key_bias[static_cast<int64_t>(b) * ld_bias + key] : 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        s.pt[tx * 4 + j][ty * 4 + i] =
            valid ? __fadd_rn(__fmul_rn(sacc[i][j], scale), bias) : -CUDART_INF_F;
    }
    __syncthreads();

    // online softmax of row sr over keys sq, sq + 4, ...: every block holds a valid key, so the
    // new maximum is finite and exp(-inf - m) = 0 starts the running sum
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) mx = fmaxf(mx, s.pt[jj * 4 + sq][sr]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float m_new = fmaxf(m_run, mx);
    const float alpha = expf(m_run - m_new);
    float part = 0.f;
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const float p = expf(s.pt[jj * 4 + sq][sr] - m_new);
      s.pt[jj * 4 + sq][sr] = p;
      part += p;
    }
    part += __shfl_xor_sync(0xffffffffu, part, 8);
    part += __shfl_xor_sync(0xffffffffu, part, 16);
    l_run = __fadd_rn(__fmul_rn(l_run, alpha), part);
    m_run = m_new;
    if (sq == 0) s.alpha[sr] = alpha;
    __syncthreads();

    // O = O * alpha + P V for rows ty*4 + i, columns tx*4 + c and 64 + tx*4 + c
    float al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) al[i] = s.alpha[ty * 4 + i];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c) o[i][c] *= al[i];
#pragma unroll 4
    for (int j = 0; j < FA32_BK; ++j) {
      const float4 p = *reinterpret_cast<const float4*>(&s.pt[j][ty * 4]);
      const float4 v0 = *reinterpret_cast<const float4*>(&s.v[j][tx * 4]);
      const float4 v1 = *reinterpret_cast<const float4*>(&s.v[j][64 + tx * 4]);
      const float pv[4] = {p.x, p.y, p.z, p.w};
      const float vr[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) o[i][c] = fmaf(pv[i], vr[c], o[i][c]);
    }
    __syncthreads();  // the next block's loads overwrite kt, v and pt
  }

  if (sq == 0) s.lsum[sr] = l_run;
  __syncthreads();
  float* ob = out + static_cast<int64_t>(b) * bs_o + h * FA32_D;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = q0 + ty * 4 + i;
    if (t >= tq) continue;
    const float l = s.lsum[ty * 4 + i];
    float r[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) r[c] = __fdiv_rn(o[i][c], l);
    if (gate != nullptr) {
      // per-(token, head) output gate (kinomlx/models/ltx2/transformer/attention.py:364-368)
      const float g = gate[static_cast<int64_t>(b) * bs_g + static_cast<int64_t>(t) * ld_g + h];
#pragma unroll
      for (int c = 0; c < 8; ++c) r[c] = __fmul_rn(r[c], g);
    }
    const float4 w0 = make_float4(r[0], r[1], r[2], r[3]);
    const float4 w1 = make_float4(r[4], r[5], r[6], r[7]);
    *reinterpret_cast<float4*>(ob + static_cast<int64_t>(t) * ld_o + tx * 4) = w0;
    *reinterpret_cast<float4*>(ob + static_cast<int64_t>(t) * ld_o + 64 + tx * 4) = w1;
  }
}

// ---------------------------------------------------------------- AdaLN
// out = norm(x) * (1 + scale[b]) + shift[b] with fp32 statistics; one CTA of 256 threads per row,
// the row in registers (dim <= 8192). norm: 0 RMS, 1 LayerNorm, 2 none.
constexpr int ADALN32_THREADS = 256;

__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum_f(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(ADALN32_THREADS)
    adaln_f32_kernel(const float* __restrict__ x, int64_t ldx, int64_t bsx,
                     const float* __restrict__ shift, const float* __restrict__ scale,
                     int64_t bs_mod, float* __restrict__ out, int64_t ldo, int64_t bso, int rows,
                     int dim, int norm, float eps) {
  __shared__ float red[8];
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x / rows;
  const int r = blockIdx.x % rows;
  const float* xr = x + static_cast<int64_t>(b) * bsx + static_cast<int64_t>(r) * ldx;
  float vals[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int c = threadIdx.x + i * ADALN32_THREADS;
    vals[i] = c < dim ? xr[c] : 0.f;
  }
  const float fdim = static_cast<float>(dim);
  float mean = 0.f, inv = 1.f;
  if (norm == 1) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) s += vals[i];
    mean = __fdiv_rn(block_sum_256(s, red), fdim);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int c = threadIdx.x + i * ADALN32_THREADS;
      const float d = vals[i] - mean;
      q += c < dim ? d * d : 0.f;
    }
    inv = rsqrtf(__fdiv_rn(block_sum_256(q, red), fdim) + eps);
  } else if (norm == 0) {
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) q += vals[i] * vals[i];
    inv = rsqrtf(__fdiv_rn(block_sum_256(q, red), fdim) + eps);
  }
  const float* sh = shift + static_cast<int64_t>(b) * bs_mod;
  const float* sc = scale + static_cast<int64_t>(b) * bs_mod;
  float* orow = out + static_cast<int64_t>(b) * bso + static_cast<int64_t>(r) * ldo;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int c = threadIdx.x + i * ADALN32_THREADS;
    if (c >= dim) continue;
    const float y = norm == 2 ? vals[i] : __fmul_rn(__fsub_rn(vals[i], mean), inv);
    orow[c] = __fadd_rn(__fmul_rn(y, __fadd_rn(1.0f, sc[c])), sh[c]);
  }
}

// ---------------------------------------------------------------- QK RMSNorm + pair RoPE
// In place on token-major x (batch x tokens x heads*128): per-head RMSNorm with a 128-entry
// weight (fp32 statistics, eps), then the adjacent-pair rotation out_e = y_e cos_e - y_o sin_e,
// out_o = y_o cos_o + y_e sin_o with fp32 tables (table_batch, table_tokens, 128), token t
// reading table row table_offset + t. One warp per (batch, token, head), four values per lane.
__global__ void __launch_bounds__(256)
    qk_norm_rope_f32_kernel(float* x, int64_t ld, int64_t bs, int tokens, int heads,
                            const float* __restrict__ weight, int per_head_norm, int rope_pairs,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            int table_batched, int64_t table_tokens, int64_t table_offset,
                            float eps, int64_t items) {
  griddep_wait();
  griddep_launch();
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (item >= items) return;
  const int lane = threadIdx.x & 31;
  const int h = static_cast<int>(item % heads);
  const int64_t bt = item / heads;
  const int t = static_cast<int>(bt % tokens);
  const int b = static_cast<int>(bt / tokens);
  float* p = x + static_cast<int64_t>(b) * bs + static_cast<int64_t>(t) * ld + h * 128 + lane * 4;
  float4 v = *reinterpret_cast<float4*>(p);
  if (per_head_norm) {
    const float ss = warp_sum_f(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
    const float4 wv = *reinterpret_cast<const float4*>(weight + lane * 4);
    v.x = __fmul_rn(__fmul_rn(v.x, inv), wv.x);
    v.y = __fmul_rn(__fmul_rn(v.y, inv), wv.y);
    v.z = __fmul_rn(__fmul_rn(v.z, inv), wv.z);
    v.w = __fmul_rn(__fmul_rn(v.w, inv), wv.w);
  }
  if (rope_pairs) {
    const int64_t row = (table_batched ? static_cast<int64_t>(b) * table_tokens : 0) + table_offset + t;
    const float4 c = *reinterpret_cast<const float4*>(cos_t + row * 128 + lane * 4);
    const float4 s = *reinterpret_cast<const float4*>(sin_t + row * 128 + lane * 4);
    float4 r;
    r.x = __fadd_rn(__fmul_rn(v.x, c.x), __fmul_rn(-v.y, s.x));
    r.y = __fadd_rn(__fmul_rn(v.y, c.y), __fmul_rn(v.x, s.y));
    r.z = __fadd_rn(__fmul_rn(v.z, c.z), __fmul_rn(-v.w, s.z));
    r.w = __fadd_rn(__fmul_rn(v.w, c.w), __fmul_rn(v.z, s.w));
    v = r;
  }
  *reinterpret_cast<float4*>(p) = v;
}

// In place on token-major x (batch x tokens x heads*128): RMSNorm over the whole row with a
// (heads*128) weight (fp32 statistics, eps), then the split-half rotation of each head
// (first, second) = (x[i], x[i + 64]) -> (first c - second s, first s + second c) with fp32
// tables (table_batch, heads, table_tokens, 64), token t reading table row table_offset + t
// (kinomlx/models/ltx2/transformer/attention.py:330-342, rope.py:18-61). One CTA of 256 threads
// per (batch, token) row; thread k holds the pairs k + 256 j (pair p = head * 64 + i).
constexpr int QKROW32_MAX_PAIRS = 16;  // per thread: rows up to 8192 wide

__global__ void __launch_bounds__(256)
    qk_norm_rope_row_f32_kernel(float* x, int64_t ld, int64_t bs, int tokens, int heads,
                                const float* __restrict__ weight, int full_row_norm,
                                int rope_split, const float* __restrict__ cos_t,
                                const float* __restrict__ sin_t, int table_batched,
                                int64_t table_tokens, int64_t table_offset, float eps) {
  __shared__ float red[8];
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x / tokens;
  const int t = blockIdx.x % tokens;
  float* row = x + static_cast<int64_t>(b) * bs + static_cast<int64_t>(t) * ld;
  const int pairs = heads * 64;
  float e1[QKROW32_MAX_PAIRS], e2[QKROW32_MAX_PAIRS];
#pragma unroll
  for (int j = 0; j < QKROW32_MAX_PAIRS; ++j) {
    const int p = threadIdx.x + j * 256;
    const int base = (p >> 6) * 128 + (p & 63);
    e1[j] = p < pairs ? row[base] : 0.f;
    e2[j] = p < pairs ? row[base + 64] : 0.f;
  }
  if (full_row_norm) {
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < QKROW32_MAX_PAIRS; ++j) q += e1[j] * e1[j] + e2[j] * e2[j];
    const float inv = rsqrtf(__fdiv_rn(block_sum_256(q, red), static_cast<float>(heads * 128)) + eps);
#pragma unroll
    for (int j = 0; j < QKROW32_MAX_PAIRS; ++j) {
      const int p = threadIdx.x + j * 256;
      if (p >= pairs) continue;
      const int base = (p >> 6) * 128 + (p & 63);
      e1[j] = __fmul_rn(__fmul_rn(e1[j], inv), weight[base]);
      e2[j] = __fmul_rn(__fmul_rn(e2[j], inv), weight[base + 64]);
    }
  }
  const int64_t trow = (table_batched ? static_cast<int64_t>(b) : 0) * heads;
#pragma unroll
  for (int j = 0; j < QKROW32_MAX_PAIRS; ++j) {
    const int p = threadIdx.x + j * 256;
    if (p >= pairs) continue;
    const int h = p >> 6, i = p & 63;
    const int base = h * 128 + i;
    float o1 = e1[j], o2 = e2[j];
    if (rope_split) {
      const int64_t entry = ((trow + h) * table_tokens + table_offset + t) * 64 + i;
      const float c = cos_t[entry], sn = sin_t[entry];
      o1 = __fsub_rn(__fmul_rn(e1[j], c), __fmul_rn(e2[j], sn));
      o2 = __fadd_rn(__fmul_rn(e1[j], sn), __fmul_rn(e2[j], c));
    }
    row[base] = o1;
    row[base + 64] = o2;
  }
}

// out[r, c] = a[r, c] + b[c] (the per-block modulation tables plus the step's timestep
// projection, kinomlx/models/ltx2/transformer/transformer.py:178-186).
__global__ void add_rows_f32_kernel(const float* __restrict__ a, const float* __restrict__ bv,
                                    float* __restrict__ out, int64_t total, int n) {
  griddep_wait();
  griddep_launch();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __fadd_rn(a[i], bv[i % n]);
}

// ---------------------------------------------------------------- elementwise
constexpr int ELEM32_GELU = 0;
constexpr int ELEM32_SILU = 1;
constexpr int ELEM32_CFG = 2;      // a = cond, b = uncond: b + s0 * (a - b)
constexpr int ELEM32_EULER_V = 3;  // a = sample, b = velocity: a + s0 * b
constexpr int ELEM32_EULER_D = 4;  // a = sample, b = denoised: b + s0 * (a - b)

__global__ void elementwise_f32_kernel(int kind, const float* a, const float* bsrc, float* out,
                                       int64_t n, float s0) {
  griddep_wait();
  griddep_launch();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = a[i];
    float y;
    switch (kind) {
      case ELEM32_GELU:
        y = gelu_tanh_exact_f32(x);
        break;
      case ELEM32_SILU:
        y = silu_exact_f32(x);
        break;
      case ELEM32_CFG: {
        const float u = bsrc[i];
        y = __fadd_rn(u, __fmul_rn(s0, __fsub_rn(x, u)));
        break;
      }
      case ELEM32_EULER_D: {
        const float d = bsrc[i];
        y = __fadd_rn(d, __fmul_rn(s0, __fsub_rn(x, d)));
        break;
      }
      default:
        y = __fadd_rn(x, __fmul_rn(s0, bsrc[i]));
        break;
    }
    out[i] = y;
  }
}

// out[b, r, c] = silu(x[b, r, c]) * x[b, r, width + c]: the gate half first, the content half
// second (kinomlx/models/flux2/transformer.py:63-65). out may alias x (each output reads only its
// own row's gate and content columns, and output column c <= input column c).
__global__ void swiglu_f32_kernel(const float* x, int64_t ldx, int64_t bsx, float* out,
                                  int64_t ldo, int64_t bso, int64_t rows, int width,
                                  int64_t total) {
  griddep_wait();
  griddep_launch();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % width);
    const int64_t br = i / width;
    const int64_t r = br % rows;
    const int64_t b = br / rows;
    const float* xr = x + b * bsx + r * ldx;
    const float g = xr[c];
    const float u = xr[width + c];
    out[b * bso + r * ldo + c] = __fmul_rn(silu_exact_f32(g), u);
  }
}

// [cos(t f_i), sin(t f_i)], f_i = exp(-ln(10000) i / (dim/2)), fp32 out (batch, dim).
__global__ void timestep_embedding_f32_kernel(const float* __restrict__ t, float* __restrict__ out,
                                              int dim) {
  griddep_wait();
  griddep_launch();
  const int half = dim / 2;
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float f = expf(__fdiv_rn(__fmul_rn(-9.210340371976184f, static_cast<float>(i)),
                                   static_cast<float>(half)));
    const float ang = __fmul_rn(t[b], f);
    out[static_cast<int64_t>(b) * dim + i] = cosf(ang);
    out[static_cast<int64_t>(b) * dim + half + i] = sinf(ang);
  }
}

// ---------------------------------------------------------------- video VAE (fp32)
// 3x3x3 convolution as an implicit GEMM on the CUDA cores: M = voxels of the un-shuffled output
// (F x H x W), N = output channels, K = 27 taps x Cin with the A rows gathered from the shifted
// input voxels under the reference's padding: temporal replicate (causal: two copies of the first
// frame in front; otherwise one at each end), spatial zero (kinomlx/models/ltx2/video_vae/
// blocks.py:97-139). 128 x 128 tiles and 8 x 8 outputs per thread as in gemm_f32_kernel; Cin % 16
// == 0 keeps every 16-wide k slice inside one tap. Epilogue: + bias, then + residual (separate
// roundings, as the reference adds them); with a depth-to-space stride the weight rows are
// sub-position-major (n = sub * C' + c) and each value is stored at its shuffled position, the
// first output frame dropped when the temporal stride is 2 (decoder.py:80-121).
struct Conv32Shape {
  int F, H, W, Cin, N;
  int causal;
  int st, sh, sw;
};

__global__ void __launch_bounds__(F32_THREADS, 2)
    conv3d_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                      const float* __restrict__ bias, const float* residual, float* out,
                      Conv32Shape s) {
  __shared__ __align__(16) float As[2][F32_BK][F32_BM + F32_PAD];
  __shared__ __align__(16) float Ws[2][F32_BK][F32_BN + F32_PAD];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int M = s.F * s.H * s.W;
  const int K = 27 * s.Cin;
  const int row0 = blockIdx.y * F32_BM;
  const int col0 = blockIdx.x * F32_BN;
  const int lr = tid >> 2;
  const int lk = (tid & 3) * 4;
  int vf[2], vh[2], vw[2];
  bool vok[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int m = row0 + lr + 64 * p;
    vok[p] = m < M;
    const int mm = vok[p] ? m : 0;
    vw[p] = mm % s.W;
    vh[p] = (mm / s.W) % s.H;
    vf[p] = mm / (s.W * s.H);
  }
  float4 ra[2], rw[2];
  auto load = [&](int k0) {
    const int tap = k0 / s.Cin;
    const int ci = k0 - tap * s.Cin + lk;
    const int kt = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      int sf = s.causal ? vf[p] + kt - 2 : vf[p] + kt - 1;
      sf = sf < 0 ? 0 : (sf > s.F - 1 ? s.F - 1 : sf);
      const int shh = vh[p] + kh - 1, sww = vw[p] + kw - 1;
      const bool in = vok[p] && shh >= 0 && shh < s.H && sww >= 0 && sww < s.W;
      ra[p] = in ? *reinterpret_cast<const float4*>(
                       x + ((static_cast<int64_t>(sf) * s.H + shh) * s.W + sww) * s.Cin + ci)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
      const int c = col0 + lr + 64 * p;
      rw[p] = c < s.N ? *reinterpret_cast<const float4*>(w + static_cast<int64_t>(c) * K + k0 + lk)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int r = lr + 64 * p;
      As[buf][lk + 0][r] = ra[p].x;
      As[buf][lk + 1][r] = ra[p].y;
      As[buf][lk + 2][r] = ra[p].z;
      As[buf][lk + 3][r] = ra[p].w;
      Ws[buf][lk + 0][r] = rw[p].x;
      Ws[buf][lk + 1][r] = rw[p].y;
      Ws[buf][lk + 2][r] = rw[p].z;
      Ws[buf][lk + 3][r] = rw[p].w;
    }
  };
  const int ty = tid >> 4;
  const int tx = tid & 15;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const int ktiles = K / F32_BK;
  load(0);
  store(0);
  __syncthreads();
  for (int t = 0; t < ktiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ktiles) load((t + 1) * F32_BK);
#pragma unroll
    for (int kk = 0; kk < F32_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Ws[buf][kk][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
    }
    if (t + 1 < ktiles) store(buf ^ 1);
    __syncthreads();
  }
  const int sub = s.st * s.sh * s.sw;
  const int Cp = s.N / sub;
  const int Ho = s.H * s.sh, Wo = s.W * s.sw;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
    const int ow0 = m % s.W, oh0 = (m / s.W) % s.H, of0 = m / (s.W * s.H);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (c >= s.N) continue;
      float v = acc[i][j];
      if (bias != nullptr) v = __fadd_rn(v, bias[c]);
      if (sub == 1) {
        const int64_t o = static_cast<int64_t>(m) * s.N + c;
        if (residual != nullptr) v = __fadd_rn(v, residual[o]);
        out[o] = v;
      } else {
        const int sp = c / Cp, cc = c - sp * Cp;
        const int dt = sp / (s.sh * s.sw), dh = (sp / s.sw) % s.sh, dw = sp % s.sw;
        const int of = of0 * s.st + dt - (s.st > 1 ? 1 : 0);
        if (of < 0) continue;
        out[((static_cast<int64_t>(of) * Ho + oh0 * s.sh + dh) * Wo + ow0 * s.sw + dw) * Cp + cc] = v;
      }
    }
  }
}

// Stepwise PixelNorm in fp32 (square, mean, + eps, sqrt, divide: kinomlx/kernels/fused_ops.py:
// 460-476), then optionally SiLU; one warp per voxel, channels % 4 == 0.
__global__ void pixel_norm_f32_kernel(const float* __restrict__ x, float* __restrict__ out,
                                      int64_t voxels, int C, float eps, int apply_silu) {
  griddep_wait();
  griddep_launch();
  const int64_t voxel = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (voxel >= voxels) return;
  const int lane = threadIdx.x & 31;
  const float* row = x + voxel * C;
  float sq = 0.f;
  for (int c = lane * 4; c < C; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(row + c);
    sq += __fmul_rn(v.x, v.x) + __fmul_rn(v.y, v.y) + __fmul_rn(v.z, v.z) + __fmul_rn(v.w, v.w);
  }
  sq = warp_sum_f(sq);
  const float rms = sqrtf(__fadd_rn(__fdiv_rn(sq, static_cast<float>(C)), eps));
  float* orow = out + voxel * C;
  for (int c = lane * 4; c < C; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(row + c);
    float y[4] = {__fdiv_rn(v.x, rms), __fdiv_rn(v.y, rms), __fdiv_rn(v.z, rms), __fdiv_rn(v.w, rms)};
    if (apply_silu) {
#pragma unroll
      for (int k = 0; k < 4; ++k) y[k] = silu_exact_f32(y[k]);
    }
    *reinterpret_cast<float4*>(orow + c) = make_float4(y[0], y[1], y[2], y[3]);
  }
}

// Affine GroupNorm(32) in fp32 with two-pass statistics (kinomlx/kernels/fused_ops.py:47-139,
// 375-409), then optionally SiLU. One CTA of 1024 threads per group walks all the group's
// elements three times (sum, squared deviations, apply); fixed-order tree reductions, so the
// result does not depend on scheduling.
constexpr int GN32_THREADS = 1024;

__device__ __forceinline__ float block_sum_1024(float v, float* red) {
  v = warp_sum_f(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = threadIdx.x < 32 ? red[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) t = warp_sum_f(t);
  if (threadIdx.x == 0) red[32] = t;
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(GN32_THREADS)
    group_norm_f32_kernel(const float* __restrict__ x, const float* __restrict__ weight,
                          const float* __restrict__ bias, float* __restrict__ out, int64_t voxels,
                          int C, float eps, int apply_silu) {
  __shared__ float red[33];
  griddep_wait();
  griddep_launch();
  const int g = blockIdx.x;
  const int gc = C / 32;
  const int64_t n = voxels * gc;
  auto addr = [&](int64_t e) { return (e / gc) * C + g * gc + (e % gc); };
  float s = 0.f;
  for (int64_t e = threadIdx.x; e < n; e += GN32_THREADS) s += x[addr(e)];
  const float mean = __fdiv_rn(block_sum_1024(s, red), static_cast<float>(n));
  float q = 0.f;
  for (int64_t e = threadIdx.x; e < n; e += GN32_THREADS) {
    const float d = __fsub_rn(x[addr(e)], mean);
    q += __fmul_rn(d, d);
  }
  const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(block_sum_1024(q, red), static_cast<float>(n)), eps));
  for (int64_t e = threadIdx.x; e < n; e += GN32_THREADS) {
    const int64_t a = addr(e);
    const int c = g * gc + static_cast<int>(e % gc);
    float y = __fmul_rn(__fsub_rn(x[a], mean), rstd);
    y = __fadd_rn(__fmul_rn(y, weight[c]), bias[c]);
    out[a] = apply_silu ? silu_exact_f32(y) : y;
  }
}

// latent (channels, voxels) -> channels-last latent * std + mean (decoder.py:227-233), fp32.
__global__ void latent_to_bfhwc_f32_kernel(const float* __restrict__ lat, const float* __restrict__ sd,
                                           const float* __restrict__ mu, float* __restrict__ out,
                                           int C, int64_t voxels) {
  griddep_wait();
  griddep_launch();
  const int64_t n = voxels * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const int64_t v = i / C;
    out[i] = __fadd_rn(__fmul_rn(lat[static_cast<int64_t>(c) * voxels + v], sd[c]), mu[c]);
  }
}

}  // namespace kino
