// bf16 GEMM on the 5th-generation tensor cores (tcgen05) with fused epilogues.
//
//   out[b, m, n] = epilogue( sum_k x[b, m, k] * w[n, k] )
//
// x rows are K-contiguous (activations), w is an nn.Linear-style (out, in) weight, so both
// operands are K-major and TMA loads them straight into 128-byte-swizzled shared memory.
// One CTA per SM runs a persistent loop over 128 x BN output tiles:
//   warp 0      TMA producer (A and B tiles, STAGES-deep ring of mbarriers)
//   warp 1      allocates tensor memory and issues tcgen05.mma (one elected thread)
//   warps 2..5  epilogue: tcgen05.ld the fp32 accumulator, apply the fused op, store bf16
// Two accumulator buffers in tensor memory let the epilogue of tile i overlap the MMAs of
// tile i+1. Nothing here uses cluster multicast.
//
// The epilogue ops restate, in one pass, the reference's separate MLX operations with their
// rounding points (kinomlx/models/flux2/transformer.py:162-164 gated residuals,
// kinomlx/kernels/fused_ops.py:27-35 tanh-GELU, kinomlx/models/flux2/sampling.py:109-113 Euler,
// kinomlx/models/ltx2/transformer/attention.py:308-315 head gates).
#pragma once
#include "kino_common.cuh"

namespace kino {

enum EpiKind : int {
  EPI_NONE = 0,
  EPI_GELU = 1,
  EPI_GATED_RESIDUAL = 2,
  EPI_EULER = 3,
  EPI_SIGMOID2 = 4,
  EPI_EULER_X0 = 5,
  EPI_SWIGLU = 6,
};

struct GemmEpi {
  int kind;
  const __nv_bfloat16* bias;      // [n] or null
  const __nv_bfloat16* residual;  // gated residual source, geometry of out
  int64_t ld_res, bs_res;
  const __nv_bfloat16* gate;      // [batch, n] (batch stride bs_gate)
  int64_t bs_gate;
  int64_t act_col_begin;          // GELU only for columns >= this
  float scalar;                   // Euler dt (fp32, rounded to bf16 as the reference does)
  const __nv_bfloat16* aux;       // Euler current sample
  int64_t ld_aux, bs_aux;
  float scalar2;                  // EULER_X0: fp32(sigma_next / sigma)
  // Per-head RMSNorm + adjacent-pair RoPE on up to two head-aligned column ranges (q and k of a
  // fused projection): range r covers [norm_col[r], norm_col[r] + norm_width) and uses the
  // 128-entry weight norm_w[r]; rows read RoPE table row rope_offset + row.
  const __nv_bfloat16* norm_w[2];
  int64_t norm_col[2];
  int64_t norm_width;
  const float* rope_cos;
  const float* rope_sin;
  int64_t rope_rows, rope_offset;
  int rope_batched;
  float norm_eps;
  // Sequence-parallel scatter (batch 1): output columns [0, scatter_cols) are stored straight
  // into the receive buffers of the GPUs that own their heads. Column c of segment
  // s = c / seg_width (q, k or v) goes to rank r = (c % seg_width) / part_width, row
  // scatter_row0 + row, column seg_slot[s] * part_width + c % part_width of scatter_ptrs[r]
  // (row stride scatter_ld). Null scatter_ptrs: every column to `out`.
  __nv_bfloat16* const* scatter_ptrs;
  int scatter_cols, seg_width, part_width;
  int64_t scatter_ld, scatter_row0;
  int seg_slot[4];
  // Rows [0, lead_rows) (batch 1, whole tiles) take the second weight (its own tensor map) and
  // these norm weights and gate: the text rows of a joint [text | image] sequence.
  int lead_rows;
  const __nv_bfloat16* norm_w_lead[2];
  const __nv_bfloat16* gate_lead;
  int bias_after_round;  // round the product to bf16 before adding the bias (packed linears)
};

// Where the 32- or 128-column chunk of output row `row` starting at col0 is stored: this GPU's
// output, or another GPU's receive buffer for scattered columns (a chunk never straddles a part:
// part widths are multiples of 128).
__device__ __forceinline__ __nv_bfloat16* gemm_dst(const GemmEpi& e, __nv_bfloat16* out,
                                                   int64_t out_off, int row, int col0) {
  if (e.scatter_ptrs != nullptr && col0 < e.scatter_cols) {
    const int seg = col0 / e.seg_width;
    const int within = col0 - seg * e.seg_width;
    const int r = within / e.part_width;
    const int c = within - r * e.part_width;
    return e.scatter_ptrs[r] + (e.scatter_row0 + row) * e.scatter_ld +
           static_cast<int64_t>(e.seg_slot[seg]) * e.part_width + c;
  }
  return out + out_off + col0;
}

struct GemmShape {
  int batch, m, n, k;
  int64_t ldo, bs_out;
  int tiles_m, tiles_n, num_tiles, kblocks;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
// Warp 0 TMA, warp 1 MMA, warps 2..9 epilogue: two warps per tensor-memory lane quarter, each
// draining half of the tile's columns, so the fused epilogues (QK norm + RoPE, GELU) finish
// within the next tile's MMAs.
constexpr int GEMM_EPI_WARPS = 8;
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;
// The implicit-GEMM conv keeps one epilogue warp per quarter.
constexpr int CONV_THREADS = 192;
// The CTA-pair conv: warp 0 TMA, warp 1 MMA, eight epilogue warps (two per TMEM lane quarter).
constexpr int CONV_PAIR_EPI_WARPS = 8;
constexpr int CONV_PAIR_THREADS = 32 * (2 + CONV_PAIR_EPI_WARPS);

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  // barriers: full[S], empty[S], tmem_full[2], tmem_empty[2], drain; then tmem base + abort
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int TOTAL = TILE_BYTES + BAR_BYTES + 1024;  // + alignment slack
};

__device__ __forceinline__ void gemm_tile_coords(const GemmShape& s, int t, int& b, int& mt,
                                                 int& nt) {
  const int per_n = s.batch * s.tiles_m;
  nt = t / per_n;
  const int rem = t - nt * per_n;
  b = rem / s.tiles_m;
  mt = rem - b * s.tiles_m;
}

// Apply the epilogue to 32 consecutive columns [col0, col0 + 32) of one output row and store.
__device__ __forceinline__ void gemm_epilogue_store(const GemmShape& s, const GemmEpi& e,
                                                    __nv_bfloat16* out, int b, int row,
                                                    int col0, const uint32_t (&acc)[32]) {
  if (row >= s.m || col0 >= s.n) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(acc[j]);
  if (e.bias != nullptr) {
    if (e.bias_after_round) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (col0 + g * 8 < s.n) {
        const uint4 raw = *reinterpret_cast<const uint4*>(e.bias + col0 + g * 8);
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(w4[q]);
          v[g * 8 + q * 2] += f.x;
          v[g * 8 + q * 2 + 1] += f.y;
        }
      }
    }
  }
  // Every reference path rounds the projection to the activation dtype first.
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);

  const int64_t out_off = static_cast<int64_t>(b) * s.bs_out + static_cast<int64_t>(row) * s.ldo;
  if (e.kind == EPI_SWIGLU && col0 >= e.act_col_begin) {
    // Weight rows were interleaved on the host in blocks of 16 gate + 16 content rows, so this
    // chunk holds gate[0..16) then content[0..16) of 16 output columns:
    // bf16(bf16(silu(gate)) * content) (kinomlx/models/flux2/transformer.py:63-65).
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = bf16_round(silu_fast_f32(v[j])) * v[16 + j];
    __nv_bfloat16* dst = out + out_off + e.act_col_begin + (col0 - e.act_col_begin) / 2;
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = pack_bf16x2(o[2 * j], o[2 * j + 1]);
    store_16(dst, w);
    return;
  }
  if (e.kind == EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j >= e.act_col_begin) v[j] = gelu_tanh_f32(v[j]);
  } else if (e.kind == EPI_SIGMOID2) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 2.0f * bf16_round(1.0f / (1.0f + expf(-v[j])));
  } else if (e.kind == EPI_GATED_RESIDUAL) {
    const __nv_bfloat16* res = e.residual + static_cast<int64_t>(b) * e.bs_res +
                               static_cast<int64_t>(row) * e.ld_res + col0;
    const __nv_bfloat16* gte =
        (row < e.lead_rows ? e.gate_lead : e.gate) + static_cast<int64_t>(b) * e.bs_gate + col0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (col0 + g * 8 < s.n) {
        const uint4 rr = *reinterpret_cast<const uint4*>(res + g * 8);
        const uint4 gg = *reinterpret_cast<const uint4*>(gte + g * 8);
        const uint32_t r4[4] = {rr.x, rr.y, rr.z, rr.w};
        const uint32_t g4[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 rf = unpack_bf16x2(r4[q]);
          const float2 gf = unpack_bf16x2(g4[q]);
          float& a0 = v[g * 8 + q * 2];
          float& a1 = v[g * 8 + q * 2 + 1];
          a0 = rf.x + bf16_round(gf.x * a0);
          a1 = rf.y + bf16_round(gf.y * a1);
        }
      }
    }
  } else if (e.kind == EPI_EULER_X0) {
    // x0 = bf16(x - sigma * v) in fp32, out = x0 + ratio * (x - x0) in fp32
    // (kinomlx/models/ltx2/transformer/wrappers.py:49-65, kinomlx/samplers/steps.py:36-70)
    const __nv_bfloat16* xs = e.aux + static_cast<int64_t>(b) * e.bs_aux +
                              static_cast<int64_t>(row) * e.ld_aux + col0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (col0 + g * 8 < s.n) {
        const uint4 xx = *reinterpret_cast<const uint4*>(xs + g * 8);
        const uint32_t x4[4] = {xx.x, xx.y, xx.z, xx.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 xf = unpack_bf16x2(x4[q]);
          const float xv[2] = {xf.x, xf.y};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float& a = v[g * 8 + q * 2 + h];
            const float x0 = bf16_round(__fsub_rn(xv[h], __fmul_rn(e.scalar, a)));
            a = __fadd_rn(x0, __fmul_rn(e.scalar2, __fsub_rn(xv[h], x0)));
          }
        }
      }
    }
  } else if (e.kind == EPI_EULER) {
    const __nv_bfloat16* xs = e.aux + static_cast<int64_t>(b) * e.bs_aux +
                              static_cast<int64_t>(row) * e.ld_aux + col0;
    const float dt = bf16_round(e.scalar);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (col0 + g * 8 < s.n) {
        const uint4 xx = *reinterpret_cast<const uint4*>(xs + g * 8);
        const uint32_t x4[4] = {xx.x, xx.y, xx.z, xx.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 xf = unpack_bf16x2(x4[q]);
          float& a0 = v[g * 8 + q * 2];
          float& a1 = v[g * 8 + q * 2 + 1];
          a0 = xf.x + bf16_round(dt * a0);
          a1 = xf.y + bf16_round(dt * a1);
        }
      }
    }
  }
  __nv_bfloat16* dst = gemm_dst(e, out, out_off, row, col0);
  uint32_t packed[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) packed[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
  store_row32(dst, packed, s.n - col0);
}

// Which norm range (0/1) holds the 128-column group starting at col, or -1.
__device__ __forceinline__ int gemm_norm_range(const GemmEpi& e, int col) {
#pragma unroll
  for (int r = 0; r < 2; ++r)
    if (e.norm_w[r] != nullptr && col >= e.norm_col[r] && col < e.norm_col[r] + e.norm_width)
      return r;
  return -1;
}

// One 128-wide head of one row: bias, rounding to bf16 (the projection's output), RMSNorm over
// the head with fp32 statistics and fp32 scale, rounding to bf16 (kinomlx/kernels/fused_ops.py
// rms_norm; kinomlx/models/flux2/transformer.py:68-75), then x * cos + perp(x) * sin on adjacent
// pairs with fp32 tables, one rounding (kinomlx/models/flux2/transformer.py:25-29).
__device__ __forceinline__ void gemm_head_chunk(const GemmEpi& e, int col, uint32_t taddr,
                                                float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (e.bias != nullptr) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 raw = *reinterpret_cast<const uint4*>(e.bias + col + g * 8);
      const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 t = unpack_bf16x2(w4[q]);
        v[g * 8 + 2 * q] += t.x;
        v[g * 8 + 2 * q + 1] += t.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
}

// Two passes over the head's accumulator columns in tensor memory (statistics, then the
// normalised, rotated store) keep 32 values live instead of 128.
__device__ __forceinline__ void gemm_epilogue_head(const GemmShape& s, const GemmEpi& e,
                                                   __nv_bfloat16* out, int b, int row, int col0,
                                                   int range, uint32_t taddr) {
  float ss = 0.0f;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    float v[32];
    gemm_head_chunk(e, col0 + c * 32, taddr + c * 32, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
  }
  // tcgen05.ld is warp-collective: every lane loads, only rows inside the product store
  const bool live = row < s.m && col0 < s.n;
  const float inv = rsqrtf(ss / 128.0f + e.norm_eps);
  const __nv_bfloat16* w = row < e.lead_rows ? e.norm_w_lead[range] : e.norm_w[range];
  // Tables are head-dim-major, (128, table columns): the 32 threads of a warp hold 32
  // consecutive rows, so each head-dim entry below is one contiguous 128-byte read.
  const int64_t trow = (e.rope_batched ? static_cast<int64_t>(b) * e.rope_rows : 0) +
                       e.rope_offset + row;
  const int64_t tstride = e.rope_rows * (e.rope_batched ? s.batch : 1);
  __nv_bfloat16* dst = gemm_dst(e, out, static_cast<int64_t>(b) * s.bs_out +
                                          static_cast<int64_t>(row) * s.ldo, row, col0);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    float v[32];
    gemm_head_chunk(e, col0 + c * 32, taddr + c * 32, v);
    if (!live) continue;
    const float* cs = e.rope_cos + trow + static_cast<int64_t>(c * 32) * tstride;
    const float* sn = e.rope_sin + trow + static_cast<int64_t>(c * 32) * tstride;
    uint32_t o16[16];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 raw = *reinterpret_cast<const uint4*>(w + c * 32 + g * 8);
      const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = g * 8 + 2 * q;
        const float2 t = unpack_bf16x2(w4[q]);
        const float x0 = bf16_round(v[j] * inv * t.x);
        const float x1 = bf16_round(v[j + 1] * inv * t.y);
        const float c0 = __ldg(cs + j * tstride), c1 = __ldg(cs + (j + 1) * tstride);
        const float s0 = __ldg(sn + j * tstride), s1 = __ldg(sn + (j + 1) * tstride);
        o16[g * 4 + q] = pack_bf16x2(__fadd_rn(__fmul_rn(x0, c0), __fmul_rn(-x1, s0)),
                                     __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1)));
      }
    }
    store_row32(dst + c * 32, o16, 32);
  }
}

__device__ __forceinline__ void gemm_epilogue_row(const GemmShape& s, const GemmEpi& e,
                                                  __nv_bfloat16* out, int b, int row, int col_base,
                                                  uint32_t taddr, int width) {
#pragma unroll 1
  for (int g = 0; g < width; g += 128) {
    const int range = gemm_norm_range(e, col_base + g);
    if (range >= 0) {
      gemm_epilogue_head(s, e, out, b, row, col_base + g, range, taddr + g);
    } else {
#pragma unroll 1
      for (int c = 0; c < 4 && g + c * 32 < width; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + g + c * 32, r);
        tmem_wait_ld();
        gemm_epilogue_store(s, e, out, b, row, col_base + g + c * 32, r);
      }
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_b_lead,
                        __nv_bfloat16* __restrict__ out,
                        const GemmShape s, const GemmEpi e) {
  using L = GemmSmem<BN, STAGES>;
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
      mbar_init(&tempty[i], GEMM_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
    tma_prefetch(&map_b_lead);
  }
  griddep_wait();  // the previous kernel has finished with its memory and tensor memory
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < s.num_tiles; t += gridDim.x) {
        int b, mt, nt;
        gemm_tile_coords(s, t, b, mt, nt);
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
          uint8_t* sa = smem + stage * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          mbar_expect_tx(&full[stage], L::STAGE_BYTES);
          tma_load_3d(sa, &map_a, &full[stage], kb * GEMM_BK, mt * GEMM_BM, b);
          tma_load_2d(sb, mt * GEMM_BM < e.lead_rows ? &map_b_lead : &map_b, &full[stage],
                      kb * GEMM_BK, nt * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Copies still in flight must land before the CTA exits: wait (bounded) on the last
      // phase armed on each stage. In a normal run these phases completed long ago.
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
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            umma_bf16(d_tmem, sdesc_k128(sa + kk * 32), sdesc_k128(sb + kk * 32), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
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
      // All issued MMAs must finish before tensor memory is released.
      umma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 200000000ull) {
      }
    }
  } else {
    // Epilogue warps 2..9. Tensor-memory lane quarter is fixed by warp id % 4; the two warps
    // of a quarter take the two column halves of a 256-wide tile (whole 128-column heads).
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int SPLIT = BN >= 256 ? 2 : 1;
    constexpr int WIDTH = BN / SPLIT;
    const int row_in_tile = quarter * 32 + static_cast<int>(lane);
    int local = 0;
    for (int t = blockIdx.x; t < s.num_tiles; t += gridDim.x, ++local) {
      int b, mt, nt;
      gemm_tile_coords(s, t, b, mt, nt);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int row = mt * GEMM_BM + row_in_tile;
      if (half < SPLIT)
        gemm_epilogue_row(s, e, out, b, row, nt * BN + half * WIDTH,
                          tmem_base + ((quarter * 32) << 16) + acc * BN + half * WIDTH, WIDTH);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    // scattered rows went to other GPUs: make them visible before the next kernel signals
    if (e.scatter_ptrs != nullptr) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace kino

namespace kino {

// ----------------------------------------------------------------------------- 2-SM variant
// The same product on CTA pairs (cluster of 2): one 256 x 256 output tile per pair per step,
// issued by the even CTA as tcgen05.mma.cta_group::2 (M = 256). Each CTA loads its 128 rows of A
// and its 128 rows of the weight (N half) into its own shared memory, 32 KB per stage instead of
// the 48 KB a 1-SM 128 x 256 tile needs, so six stages fit and each SM's operand traffic per
// tensor cycle drops by a third. TMA loads complete on the even CTA's barriers (no multicast
// loads); MMA completion is committed to both CTAs' barriers; each CTA's epilogue drains its own
// tensor memory (its 128 rows of the tile) and tells the even CTA when the accumulator is free.
template <int STAGES>
struct Gemm2SmSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;   // 16 KB: this CTA's 128 rows of A
  static constexpr int B_BYTES = 128 * GEMM_BK * 2;       // 16 KB: this CTA's 128 weight rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int TOTAL = TILE_BYTES + BAR_BYTES + 1024;
};

template <int STAGES>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_2sm_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_b_lead,
                         __nv_bfloat16* __restrict__ out, const GemmShape s, const GemmEpi e) {
  using L = Gemm2SmSmem<STAGES>;
  constexpr int BN = 256;  // pair tile width; this CTA loads BN / 2 weight rows
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
      mbar_init(&tempty[i], 2 * GEMM_EPI_WARPS);  // the epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
    tma_prefetch(&map_b_lead);
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

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = pair; t < s.num_tiles; t += pairs) {
        int b, mt, nt;
        gemm_tile_coords(s, t, b, mt, nt);
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
          uint8_t* sa = smem + stage * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          const uint32_t leader_full = smem_u32(&full[stage]) & kPairLeaderMask;
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * L::STAGE_BYTES);
          tma_load_3d_pair(sa, &map_a, leader_full, kb * GEMM_BK, mt * 256 + rank * 128, b);
          tma_load_2d_pair(sb, mt * 256 < e.lead_rows ? &map_b_lead : &map_b, leader_full,
                           kb * GEMM_BK, nt * BN + rank * 128);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // In a normal run every load was consumed by the leader's MMAs before the final cluster
      // barrier. After a timeout, give loads still in flight a bounded moment to land.
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
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            umma_bf16_pair(d_tmem, sdesc_k128(sa + kk * 32), sdesc_k128(sb + kk * 32), idesc,
                           (kb > 0 || kk > 0) ? 1u : 0u);
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
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // column half of the 256-wide tile (two heads each)
    const int row_in_tile = static_cast<int>(rank) * 128 + quarter * 32 + static_cast<int>(lane);
    const uint32_t leader_tempty0 = cluster_addr(smem_u32(&tempty[0]), 0);
    int local = 0;
    for (int t = pair; t < s.num_tiles; t += pairs, ++local) {
      int b, mt, nt;
      gemm_tile_coords(s, t, b, mt, nt);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int row = mt * 256 + row_in_tile;
      gemm_epilogue_row(s, e, out, b, row, nt * BN + half * (BN / 2),
                        tmem_base + ((quarter * 32) << 16) + acc * BN + half * (BN / 2), BN / 2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(leader_tempty0 + acc * 8);
    }
    // scattered rows went to other GPUs: make them visible before the next kernel signals
    if (e.scatter_ptrs != nullptr) __threadfence_system();
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
