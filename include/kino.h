/*
 * kino.h - C ABI of libkino_b200.so, the sm_100a (B200) kernels behind the denoise-step path of
 * KinoMLX (the Flux2-style MMDiT, the LTX-2 video DiT block and the tiled conv VAE decoder).
 *
 * Conventions
 *   - All tensors are caller-owned device pointers. The compute entry points allocate no device
 *     memory; the exceptions are kino_peer_alloc (cudaMalloc of a buffer shared with the other
 *     GPUs of a sequence-parallel group, freed by kino_peer_free) and the fixed scratch array of
 *     kino_group_norm_noalloc, which lives in the library's image rather than being allocated.
 *   - bf16 activations and weights, fp32 rope tables; "ld" is a row stride and "bs" a batch
 *     stride, both in elements. Row strides of TMA-read operands must be multiples of 8.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is asynchronous.
 *   - Every entry point returns a kino_status. KINO_ENOTSUPPORTED mirrors the reference's
 *     `applies()` refusals; there is no fallback path, so callers treat it as an error.
 *     kino_last_error() gives a one-line reason for the last failure on this thread.
 *
 * Each entry point names the reference interface (path:line inside the KinoMLX project) that it
 * replaces.
 */
#ifndef KINO_H
#define KINO_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int kino_status;
#define KINO_OK 0
#define KINO_EINVAL 1
#define KINO_ENOTSUPPORTED 2
#define KINO_ECUDA 3
#define KINO_ETIMEOUT 4

/* ABI version of this header (15); bumped on any signature change or addition. */
int kino_abi_version(void);

/* One-line description of the last error on the calling thread ("" if none). */
const char* kino_last_error(void);

/* Synchronises `stream`, then reads and clears the device-side error word that bounded waits in
 * the kernels set (KINO_ETIMEOUT if a wait gave up). Host-side counterpart of the reference's
 * per-step finiteness/status checks (kinomlx/models/flux2/sampling.py:241-244). */
kino_status kino_device_status(void* stream);

/* Number of SMs of the current device (the persistent kernels size their grids by it). */
int kino_num_sms(void);

/* ------------------------------------------------------------------ linear (GEMM) */
#define KINO_EPI_NONE 0           /* out = bf16(acc + bias) */
#define KINO_EPI_GELU 1           /* out = gelu_tanh(bf16(acc + bias)) for columns >= act_col_begin */
#define KINO_EPI_GATED_RESIDUAL 2 /* out = residual + bf16(gate[b] * bf16(acc + bias)) */
#define KINO_EPI_EULER 3          /* out = aux + bf16(bf16(scalar) * bf16(acc + bias)), fp32 add */
#define KINO_EPI_SIGMOID2 4       /* out = 2 * sigmoid(bf16(acc + bias)) */
#define KINO_EPI_EULER_X0 5       /* v = bf16(acc + bias); x0 = bf16(aux - scalar * v);
                                     out = x0 + scalar2 * (aux - x0), fp32 (LTX X0 + Euler) */
#define KINO_EPI_SWIGLU 6         /* columns >= act_col_begin: weight rows in blocks of 16 gate +
                                     16 content; out col act_col_begin + (col - act_col_begin)/2
                                     = bf16(bf16(silu(gate)) * content); earlier columns plain.
                                     Output width act_col_begin + (n - act_col_begin) / 2 */

typedef struct kino_epilogue {
  int kind;                /* KINO_EPI_* */
  const void* bias;        /* [n] bf16 or NULL */
  const void* residual;    /* GATED_RESIDUAL: bf16, may alias out */
  int64_t ld_residual;
  int64_t bs_residual;
  const void* gate;        /* GATED_RESIDUAL: [batch][n] bf16 at batch stride bs_gate */
  int64_t bs_gate;
  int64_t act_col_begin;   /* GELU: first column the activation applies to */
  float scalar;            /* EULER: dt = sigma_next - sigma (fp32) */
  const void* aux;         /* EULER, EULER_X0: current sample, bf16, geometry of out */
  int64_t ld_aux;
  int64_t bs_aux;
  float scalar2;           /* EULER_X0: fp32(sigma_next / sigma); `scalar` holds sigma */
  /* Optional fused QK norm + RoPE, independent of `kind`: for r in {0, 1} with
   * norm_weight[r] != NULL, the columns [norm_col[r], norm_col[r] + norm_width) (128-aligned,
   * 128-wide heads) are RMS-normalised per head with the 128-entry weight (fp32 statistics,
   * eps norm_eps, rounded to bf16) and rotated by adjacent pairs with the fp32 tables rope_cos /
   * rope_sin. The tables are head-dim-major, (128, T) with T = (rope_batched ? batch : 1) *
   * rope_rows: output row i of batch b reads column (rope_batched ? b : 0) * rope_rows +
   * rope_offset + i of each of the 128 table rows (kinomlx/models/flux2/transformer.py:25-29,
   * 68-75). */
  const void* norm_weight[2];
  int64_t norm_col[2];
  int64_t norm_width;
  const float* rope_cos;
  const float* rope_sin;
  int64_t rope_rows;
  int64_t rope_offset;
  int rope_batched;
  float norm_eps;
  /* Optional sequence-parallel scatter (batch 1; no counterpart in the reference, which runs
   * on one device): output columns [0, scatter_cols) are stored into other GPUs' receive
   * buffers instead of `out`. Column c of segment s = c / seg_width goes to rank
   * r = (c % seg_width) / part_width, row scatter_row0 + i, column
   * seg_slot[s] * part_width + c % part_width of scatter_ptrs[r] (a device array of `world`
   * pointers to bf16 buffers of scatter_rows rows, row stride scatter_ld). part_width is a
   * multiple of 128; columns past scatter_cols go to `out` as usual. */
  void* const* scatter_ptrs;
  int64_t world;
  int64_t scatter_cols;
  int64_t seg_width;
  int64_t part_width;
  int64_t scatter_ld;
  int64_t scatter_row0;
  int64_t scatter_rows;
  int seg_slot[4];
  /* Optional lead rows (lead_rows a multiple of 256 below m): output rows [0, lead_rows) of
   * every batch entry are computed with the weight w_lead (row stride ldw_lead, same n x k)
   * and, where used, norm_weight_lead and gate_lead (batch stride bs_gate) instead of w,
   * norm_weight and gate. One launch
   * then covers the text and image rows of a joint sequence whose two streams have their own
   * projections (kinomlx/models/flux2/transformer.py:77-117, DoubleBlock). */
  const void* w_lead;
  int64_t ldw_lead;
  int64_t lead_rows;
  const void* norm_weight_lead[2];
  const void* gate_lead;
  /* 1: the product is rounded to bf16 before the bias is added (then rounded again), as the
   * reference's packed linears do (quantized_matmul, then + bias:
   * kinomlx/models/ltx2/weights/quantization.py:32-43); 0: one rounding of acc + bias (addmm).
   * Not with the fused QK norm. */
  int bias_after_round;
} kino_epilogue;

/* out[b, i, j] = epilogue(sum_k x[b, i, k] * w[j, k]) on tcgen05 tensor cores.
 * x: batch x m x k (row stride ldx, batch stride bsx); w: n x k, row stride ldw ((out, in) layout);
 * out: batch x m x n (ldo, bso). Requires k % 8 == 0, n % 8 == 0, strides % 8 == 0.
 * Replaces kinomlx.kernels.mpp_linear.linear (kinomlx/kernels/mpp_linear.py:469-506) and the
 * MLX addmm/matmul projections of kinomlx/modeling/layers.py:8-31 and
 * kinomlx/models/ltx2/transformer/attention.py:41-51. `epi` may be NULL (plain product). */
kino_status kino_linear(const void* x, const void* w, void* out, int64_t batch, int64_t m,
                        int64_t n, int64_t k, int64_t ldx, int64_t bsx, int64_t ldw, int64_t ldo,
                        int64_t bso, const kino_epilogue* epi, void* stream);

/* Small-batch product (batch <= 4 rows): y[b, j] = sum_k act(x[b, k]) * w[j, k] + bias[j],
 * act = identity (0) or SiLU (1). Replaces the M=1 modulation/timestep projections
 * (kinomlx/models/flux2/transformer.py:223-258, kinomlx/models/ltx2/transformer/timestep.py:31-85). */
kino_status kino_gemv(const void* x, int64_t ldx, const void* w, const void* bias, void* y,
                      int64_t ldy, int64_t batch, int64_t n, int64_t k, int act, void* stream);

/* ------------------------------------------------------------------ attention */
typedef struct kino_attention_args {
  int64_t batch;
  int64_t heads;
  int64_t head_dim;        /* 64 or 128 */
  float scale;             /* softmax scale, head_dim^-0.5 in the reference */
  int n_q;                 /* 1 or 2 query segments (logically concatenated) */
  const void* q[2];
  void* out[2];            /* output of segment s, token-major, may alias q[s] */
  int64_t q_tokens[2];
  int64_t ld_q[2], bs_q[2], ld_out[2], bs_out[2];
  const void* gate[2];     /* optional (batch, tokens, heads) bf16 output gate per query segment:
                              out = bf16(bf16(attention) * gate) (LTX gated heads) */
  int64_t ld_gate[2], bs_gate[2];
  int n_kv;                /* 1 or 2 key/value segments */
  const void* k[2];
  const void* v[2];
  int64_t kv_tokens[2];
  int64_t ld_k[2], bs_k[2], ld_v[2], bs_v[2];
  /* Optional sequence-parallel return (batch 1, one query segment; no counterpart in the
   * reference): query row t belongs to rank t / rows_per_rank of `world`; its output row goes to
   * out_peers[rank] + (t % rows_per_rank) * ld_out[0] + out_col_offset + head * 128 (buffers of
   * rows_per_rank rows and out_cols columns), and with gate_peers its gate is read from
   * gate_peers[rank] at row t % rows_per_rank (stride ld_gate[0]), column
   * gate_head_offset + head. out_peers and gate_peers are device arrays of `world` pointers. */
  void* const* out_peers;
  const void* const* gate_peers;
  int64_t world;
  int64_t rows_per_rank;
  int64_t out_col_offset;
  int64_t out_cols;
  int64_t gate_head_offset;
  /* Optional additive key bias (one key segment, no peer return): key_bias[b * ld_key_bias + j]
   * (fp32, natural-log units) is added to q_i . k_j * scale before the softmax, as the
   * reference's additive attention masks are (kinomlx/models/ltx2/transformer/attention.py:164-186;
   * a padded text mask becomes 0 / -3.39e38, kinomlx/models/ltx2/transformer/preprocessing.py:85-96).
   * Rows 16-byte aligned, ld_key_bias a multiple of 4 covering kv_tokens rounded up to 4 (the
   * kernel reads whole float4s; entries past kv_tokens are ignored). Biases below -1e30 / log2(e)
   * are raised to it, so a row whose keys are all masked averages them uniformly. */
  const float* key_bias;
  int64_t ld_key_bias;
  /* Optional key split (kv_splits > 1, no key bias): each CTA takes one share of the key blocks
   * and a merge launch combines the shares' outputs by their row maxima and sums, so that a
   * call with few query tiles (sequence-parallel ranks, small batches) still fills the GPU.
   * Needs kino_attention_workspace_size(args, kv_splits) bytes of 16-byte aligned workspace. */
  int64_t kv_splits;
  void* workspace;
  int64_t workspace_bytes;
} kino_attention_args;

/* Workspace bytes kino_attention needs for `kv_splits` key shares (0 for one share; -1 for
 * invalid arguments): the shares' fp32 outputs and row statistics. No counterpart in the
 * reference (its attention is one MLX call). */
int64_t kino_attention_workspace_size(const kino_attention_args* args, int64_t kv_splits);

/* softmax(q k^T * scale) v over all key segments, per head, token-major operands.
 * Replaces MLX SDPA in the joint attention (kinomlx/models/flux2/kv.py:48-54,
 * kinomlx/models/flux2/transformer.py:35-53) and unmasked LTX attention
 * (kinomlx/models/ltx2/transformer/attention.py:144-161). */
kino_status kino_attention(const kino_attention_args* args, void* stream);

/* The reference dense kernel's contract: q (tq, heads*dim), k and v (tk, heads*dim), out like q.
 * Replaces kinomlx.models.ltx2.kernels.dense_attention.dense_attention
 * (kinomlx/models/ltx2/kernels/dense_attention.py:107-151); dim 64 or 128, as the reference's
 * kernel takes (dense_attention.py:87-104). */
kino_status kino_dense_attention(const void* q, const void* k, const void* v, void* out,
                                 int64_t tq, int64_t tk, int64_t heads, int64_t dim, void* stream);

/* ------------------------------------------------------------------ Sol-Attn (sparse) */
#define KINO_DTYPE_BF16 0
#define KINO_DTYPE_F16 1
#define KINO_DTYPE_F32 2  /* kino_strided_copy only */

typedef struct kino_sol_attention_args {
  const void* q;           /* (tokens, heads * 128) token-major, dtype below, row strides ld_* */
  const void* k;
  const void* v;
  int64_t ld_q, ld_k, ld_v;
  void* out;               /* (tokens, heads * 128), rows in the input order, the input dtype */
  int64_t ld_out;
  const void* gate;        /* optional (tokens, heads) per-head output gate, input order:
                              out = round(round(attention) * gate), as the LTX gated heads */
  int64_t ld_gate;
  int64_t tokens;          /* at most 512 blocks of 64 tokens */
  int64_t heads;
  int dtype;               /* KINO_DTYPE_BF16 or KINO_DTYPE_F16 */
  float tau;               /* routing threshold in standard deviations (finite) */
  const int32_t* order;    /* device (tokens): routing position -> input row, e.g. Morton */
  uint32_t* routes;        /* optional device (heads, blocks, ceil(blocks / 32)): receives the
                              routing mask words (bit b of row a: key block b routed for query
                              block a); NULL keeps them in the workspace */
  void* workspace;         /* kino_sol_attention_workspace_size bytes, 16-byte aligned */
  int64_t workspace_bytes;
} kino_sol_attention_args;

/* Workspace bytes of kino_sol_attention (fp16 copies of q, k, v in routing order, block means,
 * routing words, per-CTA block lists); -1 for invalid sizes. */
int64_t kino_sol_attention_workspace_size(int64_t tokens, int64_t heads);

/* Sol-Attn routed sparse attention (128-wide heads): tokens in 64-token blocks along `order`;
 * each query block attends exactly to the key blocks whose mean-key score exceeds the row's
 * mean + tau standard deviations (plus itself and both neighbours) and to every other block
 * through its mean key (score + log2 of its length) and mean value, in one softmax; operands
 * converted to fp16 (saturating), fp32 scores and accumulation. Replaces
 * kinomlx.models.ltx2.kernels.sol_attention.sol_attention
 * (kinomlx/models/ltx2/kernels/sol_attention.py:219-272, route_blocks :181-216). */
kino_status kino_sol_attention(const kino_sol_attention_args* args, void* stream);

/* ------------------------------------------------------------------ neighborhood attention */
/* Exact 3-D neighborhood attention of the LTX-2.5 diffusion video decoder: q, k, v and out are
 * contiguous (batch, frames, height, width, heads, 64) fp16, the queries already scaled; every
 * query attends to the window[0] x window[1] x window[2] keys around it, each window shifted
 * inward to stay whole at the grid's edges (on an axis of length L the window of position i
 * starts at clamp(i - K / 2, 0, L - K)); fp32 scores and softmax, the output rounded to fp16.
 * Windows odd and no larger than the grid. Replaces
 * kinomlx.models.ltx2.kernels.neighborhood_attention.neighborhood_attention
 * (kinomlx/models/ltx2/kernels/neighborhood_attention.py:170-221). */
kino_status kino_neighborhood_attention(const void* q, const void* k, const void* v, void* out,
                                        int64_t batch, int64_t frames, int64_t height,
                                        int64_t width, int64_t heads, const int32_t* window,
                                        void* stream);

/* The same with the output written as KINO_DTYPE_F16 or KINO_DTYPE_BF16 (rounded once from the
 * fp32 result): the diffusion decoder hands the attention straight to its bf16 proj product. */
kino_status kino_neighborhood_attention_ex(const void* q, const void* k, const void* v, void* out,
                                           int out_dtype, int64_t batch, int64_t frames,
                                           int64_t height, int64_t width, int64_t heads,
                                           const int32_t* window, void* stream);

/* ------------------------------------------------------------------ diffusion video decoder */
/* The qkv projection rows of a diffusion-decoder attention -> the neighborhood attention's
 * operands. qkv: (batch * frames * height * width, >= 3 * heads * 64) bf16 rows [q | k | v]
 * (bias already added) with row stride ld; q, k, v: contiguous (tokens, heads, 64) fp16. q and
 * k get a per-head RMSNorm (eps, learned bf16 weights of 64) and the decoder's absolute 3-D
 * RoPE on adjacent pairs: pairs [0, s0) rotate by the frame index, [s0, s0 + s1) by the row,
 * [s0 + s1, 32) by the column (section_pairs = host {s0, s1, s2}); q is also multiplied by
 * q_scale (head_dim^-1/2). rope_tables (fp32, device): cos_t (frames, s0), sin_t, cos_h
 * (height, s1), sin_h, cos_w (width, s2), sin_w, back to back. fp32 arithmetic, fp16 results.
 * Replaces the q/k half of NeighborhoodAttention3D._project_temporal_partition and
 * diffusion_passes.qk_norm_rope (kinomlx/models/ltx2/video_vae/diffusion_decoder.py:492-517,
 * kinomlx/models/ltx2/kernels/diffusion_passes.py:298-420). */
kino_status kino_na_qkv_prepare(const void* qkv, int64_t ld, void* q, void* k, void* v,
                                const void* q_norm_weight, const void* k_norm_weight,
                                const float* rope_tables, int64_t batch, int64_t frames,
                                int64_t height, int64_t width, int64_t heads,
                                const int32_t* section_pairs, float q_scale, float eps,
                                void* stream);

/* dst[i] = convert(src[i]) over an ndim-D index space (1 <= ndim <= 8, dimension ndim - 1
 * fastest): element offsets sum_d i_d * strides[d] on each side (a zero source stride
 * broadcasts), dtypes KINO_DTYPE_BF16 / _F16 / _F32 (round to nearest even on narrowing). The
 * decoder's pixel shuffles, spatial patchify / unpatchify, edge padding and dtype hand-offs
 * (kinomlx/models/ltx2/video_vae/diffusion_decoder.py:49-91, 283-308, 928-971). Destination
 * elements must not overlap each other or the source. */
kino_status kino_strided_copy(const void* src, int src_dtype, const int64_t* src_strides,
                              void* dst, int dst_dtype, const int64_t* dst_strides,
                              const int64_t* sizes, int ndim, void* stream);

/* ------------------------------------------------------------------ norms and rotary */
#define KINO_NORM_RMS 0
#define KINO_NORM_LAYER 1
#define KINO_NORM_NONE 2   /* modulation only: x * (1 + scale) + shift */

/* out = norm(x) * (1 + scale[b]) + shift[b], norm without affine, fp32 statistics.
 * x: batch x rows x dim (ldx, bsx); shift/scale: [batch][dim] at batch stride bs_mod.
 * Replaces kinomlx/models/flux2/transformer.py:56-60 (`normalized`, LayerNorm) and
 * kinomlx/models/ltx2/transformer/transformer.py:16-23 (`_adaln`, RMSNorm). dim <= 8192. */
kino_status kino_adaln(const void* x, int64_t ldx, int64_t bsx, const void* shift,
                       const void* scale, int64_t bs_mod, void* out, int64_t ldo, int64_t bso,
                       int64_t batch, int64_t rows, int64_t dim, int norm_kind, float eps,
                       void* stream);

/* RMSNorm over the last dimension; weight may be NULL (unweighted).
 * Replaces kinomlx.kernels.rms_norm (kinomlx/kernels/fused_ops.py:412-457). dim <= 8192. */
kino_status kino_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int64_t dim,
                          float eps, float weight_offset, void* stream);

#define KINO_QKNORM_NONE 0
#define KINO_QKNORM_PER_HEAD 1
#define KINO_QKNORM_FULL_ROW 2
#define KINO_ROPE_NONE 0
#define KINO_ROPE_PAIRS 1   /* adjacent pairs, tables [table_batch][table_tokens][128] */
#define KINO_ROPE_SPLIT 2   /* split halves, tables [table_batch][heads][table_tokens][64] */
#define KINO_ROPE_SPLIT64 3 /* split halves within 64-wide heads (two per 128 columns; heads still
                               counts 128-column groups), tables
                               [table_batch][2 * heads][table_tokens][32]; full-row norm only */

/* In place on token-major q or k (batch x tokens x heads*128, ld, bs): RMSNorm (per head or over
 * the whole row) with weight, rounded to bf16, then RoPE from fp32 tables. Token t reads table
 * row table_offset + t. Replaces QKNorm + rotate (kinomlx/models/flux2/transformer.py:17-32,
 * 68-75) and q_norm/k_norm + apply_rotary_emb
 * (kinomlx/models/ltx2/transformer/attention.py:330-342). */
kino_status kino_qk_norm_rope(void* x, int64_t ld, int64_t bs, int64_t batch, int64_t tokens,
                              int64_t heads, const void* weight, int norm_kind, int rope_kind,
                              const float* cos_table, const float* sin_table, int table_batched,
                              int64_t table_tokens, int64_t table_offset, float eps, void* stream);

/* kino_qk_norm_rope for batch 1 with the result stored into the sequence-parallel receive
 * buffers instead of in place (no counterpart in the reference, which runs on one device): head
 * h of token t goes to rank r = h / (heads / world), row dst_row0 + t, columns
 * [dst_slot * (heads / world) * 128 + (h % (heads / world)) * 128, +128) of dst_ptrs[r] (a
 * device array of `world` bf16 buffers of dst_rows rows, row stride dst_ld). */
kino_status kino_qk_norm_rope_to_peers(const void* x, int64_t ld, int64_t tokens, int64_t heads,
                                       const void* weight, int norm_kind, int rope_kind,
                                       const float* cos_table, const float* sin_table,
                                       int table_batched, int64_t table_tokens,
                                       int64_t table_offset, float eps, void* const* dst_ptrs,
                                       int64_t world, int64_t dst_ld, int64_t dst_row0,
                                       int64_t dst_rows, int64_t dst_slot, void* stream);

/* value (batch, tokens, heads*2*half) bf16, tables (table_batch, heads, tokens, half) fp32.
 * Replaces kinomlx.kernels.split_rope.rotate (kinomlx/kernels/split_rope.py:159-163) with the
 * same rounding (bit-identical to the reference graph). */
kino_status kino_split_rope(const void* x, const float* cos_table, const float* sin_table,
                            void* out, int64_t batch, int64_t tokens, int64_t heads, int64_t half,
                            int table_batched, void* stream);

/* ------------------------------------------------------------------ elementwise and sampler */
/* tanh-GELU / SiLU with fp32 opmath (kinomlx/kernels/fused_ops.py:327-372). n % 8 == 0. */
kino_status kino_gelu_tanh(const void* x, void* out, int64_t n, void* stream);
kino_status kino_silu(const void* x, void* out, int64_t n, void* stream);

/* out = uncond + guidance * (cond - uncond) in bf16 (kinomlx/models/flux2/sampling.py:264-280). */
kino_status kino_cfg_combine(const void* cond, const void* uncond, float guidance, void* out,
                             int64_t n, void* stream);

/* Klein Euler: out = bf16(f32(x) + f32(bf16(bf16(dt) * v))) (kinomlx/models/flux2/sampling.py:109-113). */
kino_status kino_euler_velocity(const void* x, const void* v, float dt, void* out, int64_t n,
                                void* stream);

/* LTX X0 + Euler: x0 = bf16(x - sigma * v) (fp32), out = bf16(x0 + ratio * (x - x0)) (fp32),
 * ratio = fp32(sigma_next / sigma) (kinomlx/models/ltx2/transformer/wrappers.py:49-65,
 * kinomlx/samplers/steps.py:36-70). */
kino_status kino_euler_x0(const void* x, const void* v, float sigma, float ratio, void* out,
                          int64_t n, void* stream);

/* Deterministic Euler on a denoised prediction: out = bf16(d + ratio * (x - d)) in fp32 with
 * ratio = fp32(sigma_next / sigma) (replaces kinomlx/samplers/steps.py:36-70 `euler_step`).
 * n % 8 == 0, 16-byte aligned operands. */
kino_status kino_euler_step(const void* sample, const void* denoised, float ratio, void* out,
                            int64_t n, void* stream);

/* Velocity Euler: out = bf16(x + bf16(delta * f32(v))), delta = fp32(sigma_next - sigma)
 * (replaces kinomlx/samplers/steps.py:8-33 `euler_velocity_step`). n % 8 == 0. */
kino_status kino_euler_velocity_step(const void* sample, const void* velocity, float delta,
                                     void* out, int64_t n, void* stream);

/* out[r, c] = bf16(a[r, c] + b[c]); a: rows x n, b: n. The per-block modulation tables plus the
 * step's timestep projection (kinomlx/models/ltx2/transformer/transformer.py:178-186). n % 8 == 0. */
kino_status kino_add_rows(const void* a, const void* b, void* out, int64_t rows, int64_t n,
                          void* stream);

/* ------------------------------------------------------------------ sequence parallelism
 * No reference counterpart (KinoMLX runs on one device): the layout steps around the all-to-all
 * of Ulysses sequence parallelism. width = heads * 128 must split into `parts` head groups. */

/* dst[j, t, :] = src[t, j*width/parts : (j+1)*width/parts]; src rows at stride ld. */
kino_status kino_heads_pack(const void* src, int64_t ld, void* dst, int64_t tokens,
                           int64_t width, int64_t parts, void* stream);

/* dst[t, j*width/parts + c] = src[j, t, c], times gate[t, head] (bf16 product) when gate is not
 * NULL (the LTX per-head gate, kinomlx/models/ltx2/transformer/attention.py:364-368). */
kino_status kino_heads_unpack(const void* src, void* dst, int64_t ld, int64_t tokens,
                             int64_t width, int64_t parts, const void* gate, int64_t ld_gate,
                             void* stream);

/* [cos(t f_i), sin(t f_i)] features, f_i = exp(-ln(10000) i / (dim/2)); t: fp32 device [batch].
 * Replaces kinomlx/models/flux2/transformer.py:238-241 and
 * kinomlx/models/ltx2/transformer/timestep.py:13-28. */
kino_status kino_timestep_embedding(const float* t, void* out, int64_t batch, int64_t dim,
                                    void* stream);

/* ------------------------------------------------------------------ quantised weights */
#define KINO_QUANT_AFFINE 0 /* w = scale * q + bias, bf16 scale and bias per group, 2/4/8 bits */
#define KINO_QUANT_MXFP8 1  /* E4M3 x E8M0 scale per 32 */
#define KINO_QUANT_MXFP4 2  /* E2M1 x E8M0 scale per 32 */
#define KINO_QUANT_NVFP4 3  /* E2M1 x E4M3 scale per 16 */

/* Dequantise a group-quantised (rows, cols) weight into bf16: `words` holds the codes packed
 * along each row, little-endian in uint32 words ((rows, cols * bits / 32)); `scales` (and, for
 * affine, `biases`) hold one value per group of `group_size` codes ((rows, cols / group_size):
 * bf16 for affine, uint8 E8M0 / E4M3 codes otherwise). out is (rows, cols), or (cols, rows) with
 * transpose_out (the reference's pretransposed weights, packed from weight.T). Float modes are
 * exact in fp32, affine is one fp32 fma; one rounding to bf16. Requires cols to be a multiple of
 * 16 and of the group size (and rows % 16 == 0 with transpose_out). Replaces the weight side of MLX's quantized_matmul as called
 * by kinomlx/models/ltx2/weights/quantization.py:26-43 (modes and groups: tensors.py:185-203). */
kino_status kino_dequantize(const void* words, const void* scales, const void* biases, void* out,
                            int64_t rows, int64_t cols, int mode, int group_size, int bits,
                            int transpose_out, void* stream);

/* ------------------------------------------------------------------ video VAE decode */
typedef struct kino_conv3d_args {
  const void* x;            /* (frames, height, width, in_channels) bf16, channels-last */
  int64_t frames, height, width, in_channels;   /* in_channels % 64 == 0 */
  const void* weight;       /* (out_channels, 3, 3, 3, in_channels) bf16 (OTHWI) */
  int64_t out_channels;
  const void* bias;         /* (out_channels) bf16 or NULL: added in bf16 after the rounding */
  const void* residual;     /* geometry of out, or NULL (no depth-to-space only) */
  void* out;                /* plain: (F, H, W, N); depth-to-space: (F*st - (st>1), H*sh, W*sw, N/(st*sh*sw)) */
  int causal;               /* 1: two copies of the first frame in front; 0: one at each end */
  int stride_t, stride_h, stride_w;  /* depth-to-space of the output; weight rows sub-position-major */
  /* Optional GroupNorm(32) statistics of the stored output for the next layer's norm
   * (kino_group_norm_from_stats): a device buffer of kino_conv3d_stats_size() bytes, its
   * capacity in records (4 per SM). Output channels per voxel 32..1024, group size dividing 32. */
  void* stats;
  int64_t stats_records;
  /* Optional split-K workspace (device, kino_conv3d_workspace_size() bytes, zero-filled once
   * before its first use; every launch leaves it ready for the next), or NULL. With it, a conv
   * whose output tiles fill less than half of the GPU splits its 27 * Cin reduction over several
   * CTAs (fp32 partial sums, added in a fixed order by the CTA that completes the tile). */
  void* workspace;
  int64_t workspace_bytes;
} kino_conv3d_args;

/* 3x3x3 convolution with temporal replicate and spatial zero padding as an implicit GEMM on
 * tcgen05 (TMA loads the shifted input boxes; no im2col buffer). Replaces Conv3dBlock and
 * WinogradConv3d (kinomlx/models/ltx2/video_vae/blocks.py:97-139,
 * kinomlx/kernels/winograd_conv3d.py:688) and the depth-to-space of
 * DepthToSpaceUpsample3d (kinomlx/models/ltx2/video_vae/decoder.py:80-121). */
kino_status kino_conv3d(const kino_conv3d_args* args, void* stream);

/* Stepwise PixelNorm over channels (+ SiLU if apply_silu), channels <= 1024.
 * Replaces kinomlx.kernels.pixel_norm / pixel_norm_fp16 (kinomlx/kernels/fused_ops.py:460-493)
 * and the silu(pixel_norm(x)) pairs of kinomlx/models/ltx2/video_vae/blocks.py:165-168. */
kino_status kino_pixel_norm(const void* x, void* out, int64_t voxels, int64_t channels, float eps,
                            int apply_silu, void* stream);

/* Bytes of device workspace kino_group_norm needs for this shape. */
int64_t kino_group_norm_workspace_size(int64_t voxels, int64_t channels);

/* Affine GroupNorm(32) on channels-last x with fp32 two-pass statistics (+ SiLU). The grid-wide
 * reduction writes partial sums into the caller's `workspace` (at least
 * kino_group_norm_workspace_size bytes). Replaces kinomlx.kernels.group_norm
 * (kinomlx/kernels/fused_ops.py:375-409). 32 <= channels <= 2048. */
kino_status kino_group_norm(const void* x, const void* weight, const void* bias, void* out,
                            int64_t voxels, int64_t channels, float eps, int apply_silu,
                            void* workspace, int64_t workspace_bytes, void* stream);

/* Bytes of the split-K workspace kino_conv3d_args.workspace takes on the current device. */
int64_t kino_conv3d_workspace_size(void);

/* Bytes of the statistics buffer kino_conv3d fills for kino_group_norm_from_stats on the current
 * device: a header, mean and rstd, and 4 records per SM of 32 x (count, mean, m2) floats. */
int64_t kino_conv3d_stats_size(void);

/* Affine GroupNorm(32) (+ SiLU) of the output of the kino_conv3d call that filled `stats`: the
 * statistics the conv's epilogue gathered (count, mean and sum of squared deviations per group,
 * merged with Chan's pairwise formula) replace the two statistics passes over x of
 * kino_group_norm, leaving one read and one write of the activation. No counterpart in the
 * reference (its GroupNorm reads x for its statistics). */
kino_status kino_group_norm_from_stats(const void* x, const void* weight, const void* bias,
                                       void* out, int64_t voxels, int64_t channels, float eps,
                                       int apply_silu, void* stats, void* stream);

/* Largest scratch kino_group_norm_noalloc can use: 80 KiB, enough for every shape
 * kino_group_norm accepts (its statistics use at most 592 partial sums per group). */
#define KINO_GROUP_NORM_NOALLOC_SCRATCH_BYTES 81920

/* kino_group_norm without a caller workspace, for callers that cannot allocate device memory:
 * hosts that own every device allocation themselves (a plugin inside a media or inference server
 * with a fixed memory budget, an allocator that hands out only tensors) or pipelines that must
 * not call cudaMalloc/cudaFree mid-run, since those calls can synchronise the device. This entry
 * point has no counterpart in the reference (MLX allocates its own temporaries).
 *
 * Its statistics scratch is one fixed array inside the library (the size above), which every GPU
 * that loads the library keeps until the process exits; nothing is allocated per call. The first
 * call on each device looks up that array's device address (cudaGetSymbolAddress) with the device
 * current; make that first call before any stream capture. A device reset (cudaDeviceReset, or a
 * primary context released and created again) unloads the array with the module: the next call
 * in the new context looks the address up again, so that call, too, belongs outside a capture.
 * Every call shares the one array and
 * leaves its contents behind: each call writes every scratch word before reading it, so no
 * clearing is needed, but calls that overlap on the GPU (for example on two streams) race on the
 * array and must be serialised by the caller. Shapes needing more scratch than the maximum are
 * refused with KINO_ENOTSUPPORTED. Same arguments and results as kino_group_norm otherwise. */
kino_status kino_group_norm_noalloc(const void* x, const void* weight, const void* bias,
                                    void* out, int64_t voxels, int64_t channels, float eps,
                                    int apply_silu, void* stream);

/* latent (channels, voxels) bf16 (BCFHW, batch 1) -> bf16(x * std + mean) channels-last.
 * Replaces PerChannelStatistics.denormalize + the BCFHW->BFHWC transpose
 * (kinomlx/models/ltx2/video_vae/decoder.py:227-233). */
kino_status kino_latent_to_bfhwc(const void* latent, const float* std_of_means,
                                 const float* mean_of_means, void* out, int64_t channels,
                                 int64_t voxels, void* stream);

/* Accumulate one decoded tile (frames, height, width, channels*patch^2) bf16 into an fp32 BCFHW
 * canvas at pixel offset (y0, x0), unpatchified and weighted by mask_h x mask_w; the masks are
 * added to the (out_height, out_width) weight canvas. Replaces the trapezoid blend of
 * kinomlx/models/ltx2/video_vae/tiling.py:1310-1330 with unpatchify (blocks.py:200-230). */
kino_status kino_tile_blend(const void* decoded, int64_t frames, int64_t height, int64_t width,
                            int64_t channels, int64_t patch, float* canvas, float* weights,
                            int64_t out_height, int64_t out_width, int64_t y0, int64_t x0,
                            const float* mask_h, const float* mask_w, void* stream);

/* canvas[p, y, x] /= max(weights[y, x], 1e-8) (kinomlx/models/ltx2/video_vae/tiling.py:1369). */
kino_status kino_blend_normalize(float* canvas, const float* weights, int64_t planes, int64_t hw,
                                 void* stream);

/* ------------------------------------------------------------------ whole blocks
 * One call per transformer block for hosts that drive the path without Python: the launch
 * sequence of the block over the entry points above, on the caller's stream, with weights,
 * activations, modulation vectors, RoPE tables and a scratch workspace all owned by the caller.
 * The results are bit-identical to the same launches issued one by one. Weights are bf16
 * (out, in) row-major, prepared once at load time as described per field. */
#define KINO_MLP_GELU_TANH 0   /* GELU-tanh MLP (BASELINE) */
#define KINO_MLP_SWIGLU 1      /* SwiGLU, gate rows first (Klein) */

typedef struct kino_flux_block_shape {
  int64_t batch;
  int64_t text_tokens;   /* Nt: rows [0, Nt) of every batch entry are text */
  int64_t image_tokens;  /* Ni: rows [Nt, Nt + Ni) are image */
  int64_t heads;         /* D = heads * 128 */
  int64_t mlp_hidden;    /* activation width entering the MLP down projection, % 32 == 0 */
  int mlp;               /* KINO_MLP_* */
  float eps;             /* LayerNorm and QK RMSNorm epsilon (1e-6 in the reference) */
} kino_flux_block_shape;

/* Pair-RoPE tables of the joint [text | image] rows, head-dim-major (128, T), T = (batched ?
 * batch : 1) * rows: row i of batch entry b reads column (batched ? b * rows : 0) + i. */
typedef struct kino_rope_tables {
  const float* cos;
  const float* sin;
  int64_t rows;
  int batched;
} kino_rope_tables;

typedef struct kino_flux_double_weights {
  const void* img_qkv;       /* (3D, D): rows [attn.to_q; attn.to_k; attn.to_v] */
  const void* txt_qkv;       /* (3D, D): rows [attn.add_q_proj; add_k_proj; add_v_proj] */
  const void* to_out;        /* (D, D) attn.to_out.0 */
  const void* to_add_out;    /* (D, D) attn.to_add_out */
  const void* norm_q;        /* (128) attn.norm_q, norm_k, norm_added_q, norm_added_k */
  const void* norm_k;
  const void* norm_added_q;
  const void* norm_added_k;
  const void* ff_in;         /* (mlp_in, D) ff.linear_in (SwiGLU: rows in blocks of 16 gate +
                                16 content, the KINO_EPI_SWIGLU order) */
  const void* ff_out;        /* (D, mlp_hidden) ff.linear_out */
  const void* ffc_in;        /* the text stream's ff_context.linear_in / linear_out */
  const void* ffc_out;
} kino_flux_double_weights;

typedef struct kino_flux_single_weights {
  const void* fused;         /* (3D + mlp_in, D): attn.to_qkv_mlp_proj with its row blocks
                                reordered [k; v; q; mlp] (SwiGLU mlp rows interleaved as above) */
  const void* to_out;        /* (D, D + mlp_hidden) attn.to_out */
  const void* norm_q;        /* (128) */
  const void* norm_k;
} kino_flux_single_weights;

/* Bytes of workspace a double or single block of this shape needs (-1 for an invalid shape). */
int64_t kino_flux_block_workspace_size(const kino_flux_block_shape* shape);

/* One Flux2 DoubleBlock in place on hidden (B, Nt + Ni, D) bf16, text rows then image rows.
 * modulation: (B, 12 D) bf16 at batch stride bs_modulation (0: one vector for every entry),
 * the image stream's [shift, scale, gate, ff_shift, ff_scale, ff_gate] then the text stream's.
 * Replaces DoubleBlock / DoubleAttention (kinomlx/models/flux2/transformer.py:88-167). */
kino_status kino_flux_double_block(const kino_flux_block_shape* shape,
                                   const kino_flux_double_weights* weights, void* hidden,
                                   const void* modulation, int64_t bs_modulation,
                                   const kino_rope_tables* rope, void* workspace,
                                   int64_t workspace_bytes, void* stream);

/* One Flux2 SingleBlock in place on hidden (B, Nt + Ni, D); modulation (B, 3 D):
 * [shift, scale, gate]. Replaces SingleBlock / SingleAttention
 * (kinomlx/models/flux2/transformer.py:170-220). */
kino_status kino_flux_single_block(const kino_flux_block_shape* shape,
                                   const kino_flux_single_weights* weights, void* hidden,
                                   const void* modulation, int64_t bs_modulation,
                                   const kino_rope_tables* rope, void* workspace,
                                   int64_t workspace_bytes, void* stream);

typedef struct kino_ltx_block_shape {
  int64_t batch;
  int64_t tokens;          /* video tokens T */
  int64_t context_tokens;  /* text tokens Tc */
  int64_t heads;           /* D = heads * 128 */
  int64_t context_dim;     /* width of the text context (= D) */
  int64_t ff_hidden;       /* feed-forward width (4 D) */
  float eps;               /* RMSNorm epsilon (1e-6) */
} kino_ltx_block_shape;

typedef struct kino_ltx_video_block_weights {
  const void* qkv_w;       /* (3D, D): rows [attn1.to_v; attn1.to_q; attn1.to_k]; bias (3D) */
  const void* qkv_b;
  const void* g1_w;        /* (heads, D) attn1.to_gate_logits and its bias */
  const void* g1_b;
  const void* o1_w;        /* (D, D) attn1.to_out and bias */
  const void* o1_b;
  const void* qn1;         /* (D) attn1.q_norm / k_norm */
  const void* kn1;
  const void* q2_w;        /* (D, D) attn2.to_q and bias */
  const void* q2_b;
  const void* kv2_w;       /* (2D, context_dim): rows [attn2.to_k; attn2.to_v]; bias (2D) */
  const void* kv2_b;
  const void* g2_w;        /* attn2.to_gate_logits, to_out, q_norm, k_norm as above */
  const void* g2_b;
  const void* o2_w;
  const void* o2_b;
  const void* qn2;
  const void* kn2;
  const void* ff_in_w;     /* (ff_hidden, D) ff.project_in.proj and bias */
  const void* ff_in_b;
  const void* ff_out_w;    /* (D, ff_hidden) ff.project_out and bias */
  const void* ff_out_b;
} kino_ltx_video_block_weights;

/* Bytes of workspace kino_ltx_video_block needs (-1 for an invalid shape). */
int64_t kino_ltx_video_block_workspace_size(const kino_ltx_block_shape* shape);

/* One LTX-2 video block in place on hidden (B, T, D): gated self-attention (full-row QK RMSNorm,
 * split RoPE from the (1|B, heads, T, 64) fp32 tables rope_cos / rope_sin), gated text
 * cross-attention on the prompt-modulated context (B, Tc, D), GELU feed-forward, AdaLN-modulated
 * gated residuals. values: (B, 9 D) = the block's scale_shift_table plus the step's timestep
 * projection, rows (shift, scale, gate) x {attention, feed-forward} then (shift, scale, gate) of
 * the cross-attention query; prompt: (B, 2 D) = prompt_scale_shift_table plus the prompt
 * timestep projection, (shift, scale). Replaces the video path of BasicAVTransformerBlock
 * (kinomlx/models/ltx2/transformer/transformer.py:16-45, 178-276) with its Attention
 * (attention.py:249-371) and FeedForward (feed_forward.py:11-100). */
kino_status kino_ltx_video_block(const kino_ltx_block_shape* shape,
                                 const kino_ltx_video_block_weights* weights, void* hidden,
                                 const void* context, const void* values, int64_t bs_values,
                                 const void* prompt, int64_t bs_prompt, const float* rope_cos,
                                 const float* rope_sin, int rope_batched, void* workspace,
                                 int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ fp32 parity mode
 * The Flux2 block operators in single precision on the CUDA cores, for the reference's fp32
 * graph (MLX arrays in float32; BASELINE's fp32 gate is a per-op max relative error <= 1e-4).
 * Every product and sum is fp32; where the reference's graph has separate operations the
 * results are rounded separately (no fused multiply-add in the epilogues). Tensors are float*,
 * strides in elements, row strides multiples of 4 with 16-byte aligned operands. */

typedef struct kino_epilogue_f32 {
  int kind;                /* KINO_EPI_NONE, _GELU, _GATED_RESIDUAL, _EULER, _SIGMOID2 or _EULER_X0 */
  const float* bias;       /* [n] or NULL: acc + bias */
  const float* residual;   /* GATED_RESIDUAL: out = residual + gate[b] * (acc + bias); may alias out */
  int64_t ld_residual;
  int64_t bs_residual;
  const float* gate;       /* GATED_RESIDUAL: [batch][n] at batch stride bs_gate */
  int64_t bs_gate;
  int64_t act_col_begin;   /* GELU: tanh-GELU (inner clamped to +-10) on columns >= act_col_begin */
  float scalar;            /* EULER: out = aux + scalar * (acc + bias); EULER_X0: sigma */
  const float* aux;        /* EULER, EULER_X0: current sample, geometry of out; may alias out */
  int64_t ld_aux;
  int64_t bs_aux;
  float scalar2;           /* EULER_X0: v = acc + bias; x0 = aux - scalar * v;
                              out = x0 + scalar2 * (aux - x0) (scalar2 = sigma_next / sigma).
                              SIGMOID2 needs no operand: out = 2 * sigmoid(acc + bias) */
} kino_epilogue_f32;

/* kino_linear in fp32: out[b, i, j] = epilogue(sum_k x[b, i, k] * w[j, k]); w (n, k) row-major.
 * k % 4 == 0. x and w must not overlap out. Replaces the fp32 case of kinomlx.kernels.mpp_linear
 * .linear / mx.addmm (kinomlx/kernels/mpp_linear.py:469-506, kinomlx/modeling/layers.py:8-31),
 * with the gated residual of kinomlx/models/flux2/transformer.py:159-167 and the Euler update of
 * kinomlx/models/flux2/sampling.py:109-113 in the epilogue. */
kino_status kino_linear_f32(const float* x, const float* w, float* out, int64_t batch, int64_t m,
                            int64_t n, int64_t k, int64_t ldx, int64_t bsx, int64_t ldw,
                            int64_t ldo, int64_t bso, const kino_epilogue_f32* epi, void* stream);

/* softmax(q k^T * scale + key_bias) v per (batch, head), head_dim 128, token-major q (q_tokens
 * rows), k and v (kv_tokens rows); out like q and may alias it. With `gate` (batch, q_tokens,
 * heads) at row stride ld_gate and batch stride bs_gate, each head's output is multiplied by its
 * gate. `key_bias` (optional, fp32, row b at b * ld_key_bias) is an additive mask over the keys
 * (kinomlx/models/ltx2/transformer/attention.py:164-186).
 * Replaces MLX SDPA in fp32 (kinomlx/models/flux2/kv.py:48-54, kinomlx/models/flux2/
 * transformer.py:35-53, kinomlx/models/ltx2/transformer/attention.py:144-161, 364-368). */
kino_status kino_attention_f32(const float* q, const float* k, const float* v, float* out,
                               int64_t batch, int64_t heads, int64_t q_tokens, int64_t kv_tokens,
                               int64_t ld_q, int64_t bs_q, int64_t ld_k, int64_t bs_k,
                               int64_t ld_v, int64_t bs_v, int64_t ld_out, int64_t bs_out,
                               float scale, const float* gate, int64_t ld_gate, int64_t bs_gate,
                               const float* key_bias, int64_t ld_key_bias, void* stream);

/* kino_adaln in fp32: out = norm(x) * (1 + scale[b]) + shift[b], dim <= 8192
 * (kinomlx/models/flux2/transformer.py:56-60). */
kino_status kino_adaln_f32(const float* x, int64_t ldx, int64_t bsx, const float* shift,
                           const float* scale, int64_t bs_mod, float* out, int64_t ldo,
                           int64_t bso, int64_t batch, int64_t rows, int64_t dim, int norm_kind,
                           float eps, void* stream);

/* kino_qk_norm_rope in fp32, in place, in one of two forms: KINO_QKNORM_PER_HEAD (or NONE) then
 * KINO_ROPE_PAIRS (or NONE) with token-major tables (table_batch, table_tokens, 128), replacing
 * QKNorm + rotate (kinomlx/models/flux2/transformer.py:17-32, 68-75); or KINO_QKNORM_FULL_ROW (or
 * NONE) then KINO_ROPE_SPLIT (or NONE) with tables (table_batch, heads, table_tokens, 64), rows
 * up to 8192 wide, replacing q_norm/k_norm + apply_split_rotary_emb
 * (kinomlx/models/ltx2/transformer/attention.py:330-342). */
kino_status kino_qk_norm_rope_f32(float* x, int64_t ld, int64_t bs, int64_t batch,
                                  int64_t tokens, int64_t heads, const float* weight,
                                  int norm_kind, int rope_kind, const float* cos_table,
                                  const float* sin_table, int table_batched, int64_t table_tokens,
                                  int64_t table_offset, float eps, void* stream);

/* out[r, c] = a[r, c] + b[c], fp32 (kinomlx/models/ltx2/transformer/transformer.py:178-186). */
kino_status kino_add_rows_f32(const float* a, const float* b, float* out, int64_t rows, int64_t n,
                              void* stream);

/* fp32 tanh-GELU and SiLU (kinomlx/kernels/fused_ops.py:27-45, 327-372). */
kino_status kino_gelu_tanh_f32(const float* x, float* out, int64_t n, void* stream);
kino_status kino_silu_f32(const float* x, float* out, int64_t n, void* stream);

/* out = uncond + guidance * (cond - uncond) (kinomlx/models/flux2/sampling.py:264-280). */
kino_status kino_cfg_combine_f32(const float* cond, const float* uncond, float guidance,
                                 float* out, int64_t n, void* stream);

/* out = x + dt * v (kinomlx/models/flux2/sampling.py:109-113 with the model dtype fp32). */
kino_status kino_euler_velocity_f32(const float* x, const float* v, float dt, float* out,
                                    int64_t n, void* stream);

/* out = d + ratio * (x - d) in fp32 (kinomlx/samplers/steps.py:36-70 with an fp32 sample). */
kino_status kino_euler_step_f32(const float* sample, const float* denoised, float ratio,
                               float* out, int64_t n, void* stream);

/* out[b, r, c] = silu(x[b, r, c]) * x[b, r, width + c], gate half first
 * (kinomlx/models/flux2/transformer.py:63-65); out may alias x. */
kino_status kino_swiglu_f32(const float* x, int64_t ldx, int64_t bsx, float* out, int64_t ldo,
                            int64_t bso, int64_t batch, int64_t rows, int64_t width,
                            void* stream);

/* kino_timestep_embedding with fp32 features (kinomlx/models/flux2/transformer.py:238-241). */
kino_status kino_timestep_embedding_f32(const float* t, float* out, int64_t batch, int64_t dim,
                                        void* stream);

/* Video VAE decode in fp32 (same layouts as the bf16 entry points, float* tensors). */

/* kino_conv3d in fp32: x (frames, height, width, in_channels) channels-last, weight (out_channels,
 * 3, 3, 3, in_channels) OTHWI, bias (out_channels) or NULL, residual (geometry of out, no
 * depth-to-space) or NULL; out (F, H, W, N), or with strides (st, sh, sw) in {1, 2}
 * (F*st - (st > 1), H*sh, W*sw, N/(st*sh*sw)) with the weight rows sub-position-major.
 * in_channels % 16 == 0. out = conv + bias, then + residual. Replaces Conv3dBlock and the
 * depth-to-space upsample (kinomlx/models/ltx2/video_vae/blocks.py:97-139, decoder.py:80-121). */
kino_status kino_conv3d_f32(const float* x, int64_t frames, int64_t height, int64_t width,
                            int64_t in_channels, const float* weight, int64_t out_channels,
                            const float* bias, const float* residual, float* out, int causal,
                            int stride_t, int stride_h, int stride_w, void* stream);

/* Stepwise PixelNorm (+ SiLU) in fp32, channels % 4 == 0 (kinomlx/kernels/fused_ops.py:460-476). */
kino_status kino_pixel_norm_f32(const float* x, float* out, int64_t voxels, int64_t channels,
                                float eps, int apply_silu, void* stream);

/* Affine GroupNorm(32) (+ SiLU) in fp32 with two-pass statistics; needs no workspace
 * (kinomlx/kernels/fused_ops.py:375-409). */
kino_status kino_group_norm_f32(const float* x, const float* weight, const float* bias, float* out,
                                int64_t voxels, int64_t channels, float eps, int apply_silu,
                                void* stream);

/* kino_latent_to_bfhwc in fp32 (kinomlx/models/ltx2/video_vae/decoder.py:227-233). */
kino_status kino_latent_to_bfhwc_f32(const float* latent, const float* std_of_means,
                                     const float* mean_of_means, float* out, int64_t channels,
                                     int64_t voxels, void* stream);

/* kino_tile_blend with an fp32 decoded tile (kinomlx/models/ltx2/video_vae/tiling.py:1310-1330). */
kino_status kino_tile_blend_f32(const float* decoded, int64_t frames, int64_t height, int64_t width,
                                int64_t channels, int64_t patch, float* canvas, float* weights,
                                int64_t out_height, int64_t out_width, int64_t y0, int64_t x0,
                                const float* mask_h, const float* mask_w, void* stream);

/* ------------------------------------------------------------------ peer memory (NVLink)
 * Buffers that the other GPUs of a sequence-parallel group map (CUDA IPC) and write into: the
 * q/k/v receive buffers, the projection outputs the attention returns its rows to, and the
 * barrier flags. No counterpart in the reference (one device). */
typedef struct kino_ipc_handle {
  unsigned char bytes[64];
} kino_ipc_handle;

/* cudaMalloc `bytes` (zero-filled) and export an IPC handle for it. */
kino_status kino_peer_alloc(int64_t bytes, void** ptr, kino_ipc_handle* handle);
kino_status kino_peer_free(void* ptr);
/* Map another process's buffer (same node) into this process; close with kino_peer_close. */
kino_status kino_peer_open(const kino_ipc_handle* handle, void** ptr);
kino_status kino_peer_close(void* ptr);

/* Arrival barrier number `epoch` (1, 2, ...) across `world` GPUs (world <= 32): flags is a
 * device array of `world` pointers to each rank's `world` uint32 flags (zero-initialised). Rank
 * `rank` publishes its earlier stores, marks its arrival in every rank's flags and waits (at most
 * 2 s, then KINO_ETIMEOUT in kino_device_status) until every rank has arrived. */
kino_status kino_peer_barrier(void* const* flags, int64_t rank, int64_t world, int64_t epoch,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KINO_H */
