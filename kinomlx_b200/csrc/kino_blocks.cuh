// Whole transformer blocks behind one C call each: the host-side launch sequence of a Flux2
// double block, a Flux2 single block and an LTX-2 video block over the kernels of this library,
// for hosts that drive the path without Python. Every launch goes to the caller's stream in the
// order the Python model classes issue them, so the results are the same bits. Included at the
// end of kino_capi.cu (it calls the entry points defined there and shares its error state).

namespace {

constexpr int64_t kBlockAlign = 256;

int64_t align_up(int64_t v) { return (v + kBlockAlign - 1) / kBlockAlign * kBlockAlign; }

// Carves bf16 sections out of a caller workspace in order.
struct Carve {
  unsigned char* base;
  int64_t used;
  __nv_bfloat16* take(int64_t elems) {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(base + used);
    used += align_up(elems * static_cast<int64_t>(sizeof(__nv_bfloat16)));
    return p;
  }
};

bool flux_shape_ok(const kino_flux_block_shape* s, const char* who) {
  if (s == nullptr) {
    fail(KINO_EINVAL, "%s: null shape", who);
    return false;
  }
  if (s->batch < 1 || s->text_tokens < 0 || s->image_tokens < 0 ||
      s->text_tokens + s->image_tokens < 1 || s->heads < 1 || s->mlp_hidden < 32 ||
      s->mlp_hidden % 32 || (s->mlp != KINO_MLP_GELU_TANH && s->mlp != KINO_MLP_SWIGLU)) {
    fail(KINO_EINVAL, "%s: invalid shape", who);
    return false;
  }
  return true;
}

int64_t flux_mlp_in(const kino_flux_block_shape* s) {
  return s->mlp == KINO_MLP_SWIGLU ? 2 * s->mlp_hidden : s->mlp_hidden;
}

int flux_act_kind(const kino_flux_block_shape* s) {
  return s->mlp == KINO_MLP_SWIGLU ? kino::EPI_SWIGLU : kino::EPI_GELU;
}

kino_epilogue plain_epi(int kind) {
  kino_epilogue e;
  std::memset(&e, 0, sizeof(e));
  e.kind = kind;
  return e;
}

void set_gated(kino_epilogue* e, void* residual, int64_t ld, int64_t bs, const void* gate,
               int64_t bs_gate) {
  e->kind = kino::EPI_GATED_RESIDUAL;
  e->residual = residual;
  e->ld_residual = ld;
  e->bs_residual = bs;
  e->gate = gate;
  e->bs_gate = bs_gate;
}

void set_qk(kino_epilogue* e, const void* w0, int64_t col0, const void* w1, int64_t col1,
            int64_t width, const kino_rope_tables* rope, int64_t offset, float eps) {
  e->norm_weight[0] = w0;
  e->norm_col[0] = col0;
  e->norm_weight[1] = w1;
  e->norm_col[1] = col1;
  e->norm_width = width;
  e->rope_cos = rope->cos;
  e->rope_sin = rope->sin;
  e->rope_rows = rope->rows;
  e->rope_offset = offset;
  e->rope_batched = rope->batched;
  e->norm_eps = eps;
}

kino_attention_args self_attention(int64_t batch, int64_t heads, int64_t tokens, const void* q,
                                   const void* k, const void* v, void* out, int64_t ld,
                                   int64_t bs) {
  kino_attention_args a;
  std::memset(&a, 0, sizeof(a));
  a.batch = batch;
  a.heads = heads;
  a.head_dim = 128;
  a.scale = 0.08838834764831845f;  // 128^-0.5
  a.n_q = 1;
  a.q[0] = q;
  a.out[0] = out;
  a.q_tokens[0] = tokens;
  a.ld_q[0] = a.ld_out[0] = ld;
  a.bs_q[0] = a.bs_out[0] = bs;
  a.n_kv = 1;
  a.k[0] = k;
  a.v[0] = v;
  a.kv_tokens[0] = tokens;
  a.ld_k[0] = a.ld_v[0] = ld;
  a.bs_k[0] = a.bs_v[0] = bs;
  return a;
}

#define KINO_TRY(call)                  \
  do {                                  \
    const kino_status st_ = (call);     \
    if (st_ != KINO_OK) return st_;     \
  } while (0)

}  // namespace

extern "C" {

int64_t kino_flux_block_workspace_size(const kino_flux_block_shape* s) {
  if (!flux_shape_ok(s, "kino_flux_block_workspace_size")) return -1;
  const int64_t rows = s->batch * (s->text_tokens + s->image_tokens);
  const int64_t d = s->heads * 128;
  const int64_t two = 2;
  const int64_t dbl = align_up(rows * 3 * d * two) + align_up(rows * s->mlp_hidden * two);
  const int64_t sgl = align_up(rows * (3 * d + s->mlp_hidden) * two);
  return align_up(rows * d * two) + (dbl > sgl ? dbl : sgl);
}

kino_status kino_flux_double_block(const kino_flux_block_shape* s,
                                   const kino_flux_double_weights* w, void* hidden,
                                   const void* modulation, int64_t bs_modulation,
                                   const kino_rope_tables* rope, void* workspace,
                                   int64_t workspace_bytes, void* stream) {
  if (!flux_shape_ok(s, "kino_flux_double_block")) return KINO_EINVAL;
  if (w == nullptr || hidden == nullptr || modulation == nullptr || rope == nullptr ||
      workspace == nullptr)
    return fail(KINO_EINVAL, "kino_flux_double_block: null argument");
  if (s->text_tokens < 1 || s->image_tokens < 1)
    return fail(KINO_EINVAL, "kino_flux_double_block: both streams need tokens");
  if (workspace_bytes < kino_flux_block_workspace_size(s) || !aligned16(workspace))
    return fail(KINO_EINVAL, "kino_flux_double_block: workspace below %lld bytes or unaligned",
                (long long)kino_flux_block_workspace_size(s));
  const int64_t b = s->batch, nt = s->text_tokens, ni = s->image_tokens, n = nt + ni;
  const int64_t d = s->heads * 128, hid_w = s->mlp_hidden, mlp_in = flux_mlp_in(s);
  const int act = flux_act_kind(s);
  const float eps = s->eps;
  Carve c{static_cast<unsigned char*>(workspace), 0};
  __nv_bfloat16* nrm = c.take(b * n * d);
  __nv_bfloat16* qkv = c.take(b * n * 3 * d);
  __nv_bfloat16* hid = c.take(b * n * hid_w);
  __nv_bfloat16* x = static_cast<__nv_bfloat16*>(hidden);
  const __nv_bfloat16* mod = static_cast<const __nv_bfloat16*>(modulation);
  auto m = [&](int base, int j) { return mod + (base + j) * d; };  // image base 0, text base 6
  const int64_t bsx = n * d, bsq = n * 3 * d, bsh = n * hid_w;
  auto adaln = [&](int64_t r0, int64_t rows, const __nv_bfloat16* shift,
                   const __nv_bfloat16* scale) {
    return kino_adaln(x + r0 * d, d, bsx, shift, scale, bs_modulation, nrm + r0 * d, d, bsx, b,
                      rows, d, KINO_NORM_LAYER, eps, stream);
  };
  KINO_TRY(adaln(nt, ni, m(0, 0), m(0, 1)));
  KINO_TRY(adaln(0, nt, m(6, 0), m(6, 1)));
  const bool joint = nt % 256 == 0;
  if (joint) {  // text rows as lead rows: one launch per projection over both streams
    kino_epilogue e = plain_epi(kino::EPI_NONE);
    set_qk(&e, w->norm_q, 0, w->norm_k, d, d, rope, 0, eps);
    e.w_lead = w->txt_qkv;
    e.ldw_lead = d;
    e.lead_rows = nt;
    e.norm_weight_lead[0] = w->norm_added_q;
    e.norm_weight_lead[1] = w->norm_added_k;
    KINO_TRY(kino_linear(nrm, w->img_qkv, qkv, b, n, 3 * d, d, d, bsx, d, 3 * d, bsq, &e, stream));
  } else {
    kino_epilogue e = plain_epi(kino::EPI_NONE);
    set_qk(&e, w->norm_q, 0, w->norm_k, d, d, rope, nt, eps);
    KINO_TRY(kino_linear(nrm + nt * d, w->img_qkv, qkv + nt * 3 * d, b, ni, 3 * d, d, d, bsx, d,
                         3 * d, bsq, &e, stream));
    kino_epilogue et = plain_epi(kino::EPI_NONE);
    set_qk(&et, w->norm_added_q, 0, w->norm_added_k, d, d, rope, 0, eps);
    KINO_TRY(kino_linear(nrm, w->txt_qkv, qkv, b, nt, 3 * d, d, d, bsx, d, 3 * d, bsq, &et, stream));
  }
  kino_attention_args att = self_attention(b, s->heads, n, qkv, qkv + d, qkv + 2 * d, qkv,
                                           3 * d, bsq);
  KINO_TRY(kino_attention(&att, stream));
  if (joint) {
    kino_epilogue e = plain_epi(kino::EPI_NONE);
    set_gated(&e, x, d, bsx, m(0, 2), bs_modulation);
    e.w_lead = w->to_add_out;
    e.ldw_lead = d;
    e.lead_rows = nt;
    e.gate_lead = m(6, 2);
    KINO_TRY(kino_linear(qkv, w->to_out, x, b, n, d, d, 3 * d, bsq, d, d, bsx, &e, stream));
    KINO_TRY(adaln(nt, ni, m(0, 3), m(0, 4)));
    KINO_TRY(adaln(0, nt, m(6, 3), m(6, 4)));
    kino_epilogue ea = plain_epi(act);
    ea.w_lead = w->ffc_in;
    ea.ldw_lead = d;
    ea.lead_rows = nt;
    KINO_TRY(kino_linear(nrm, w->ff_in, hid, b, n, mlp_in, d, d, bsx, d, hid_w, bsh, &ea, stream));
    kino_epilogue eo = plain_epi(kino::EPI_NONE);
    set_gated(&eo, x, d, bsx, m(0, 5), bs_modulation);
    eo.w_lead = w->ffc_out;
    eo.ldw_lead = hid_w;
    eo.lead_rows = nt;
    eo.gate_lead = m(6, 5);
    KINO_TRY(kino_linear(hid, w->ff_out, x, b, n, d, hid_w, hid_w, bsh, hid_w, d, bsx, &eo, stream));
    return KINO_OK;
  }
  kino_epilogue ei = plain_epi(kino::EPI_NONE);
  set_gated(&ei, x + nt * d, d, bsx, m(0, 2), bs_modulation);
  KINO_TRY(kino_linear(qkv + nt * 3 * d, w->to_out, x + nt * d, b, ni, d, d, 3 * d, bsq, d, d,
                       bsx, &ei, stream));
  kino_epilogue et = plain_epi(kino::EPI_NONE);
  set_gated(&et, x, d, bsx, m(6, 2), bs_modulation);
  KINO_TRY(kino_linear(qkv, w->to_add_out, x, b, nt, d, d, 3 * d, bsq, d, d, bsx, &et, stream));
  kino_epilogue ea = plain_epi(act);
  kino_epilogue eo = plain_epi(kino::EPI_NONE);
  KINO_TRY(adaln(nt, ni, m(0, 3), m(0, 4)));
  KINO_TRY(kino_linear(nrm + nt * d, w->ff_in, hid + nt * hid_w, b, ni, mlp_in, d, d, bsx, d,
                       hid_w, bsh, &ea, stream));
  set_gated(&eo, x + nt * d, d, bsx, m(0, 5), bs_modulation);
  KINO_TRY(kino_linear(hid + nt * hid_w, w->ff_out, x + nt * d, b, ni, d, hid_w, hid_w, bsh,
                       hid_w, d, bsx, &eo, stream));
  KINO_TRY(adaln(0, nt, m(6, 3), m(6, 4)));
  KINO_TRY(kino_linear(nrm, w->ffc_in, hid, b, nt, mlp_in, d, d, bsx, d, hid_w, bsh, &ea, stream));
  set_gated(&eo, x, d, bsx, m(6, 5), bs_modulation);
  return kino_linear(hid, w->ffc_out, x, b, nt, d, hid_w, hid_w, bsh, hid_w, d, bsx, &eo, stream);
}

kino_status kino_flux_single_block(const kino_flux_block_shape* s,
                                   const kino_flux_single_weights* w, void* hidden,
                                   const void* modulation, int64_t bs_modulation,
                                   const kino_rope_tables* rope, void* workspace,
                                   int64_t workspace_bytes, void* stream) {
  if (!flux_shape_ok(s, "kino_flux_single_block")) return KINO_EINVAL;
  if (w == nullptr || hidden == nullptr || modulation == nullptr || rope == nullptr ||
      workspace == nullptr)
    return fail(KINO_EINVAL, "kino_flux_single_block: null argument");
  if (workspace_bytes < kino_flux_block_workspace_size(s) || !aligned16(workspace))
    return fail(KINO_EINVAL, "kino_flux_single_block: workspace below %lld bytes or unaligned",
                (long long)kino_flux_block_workspace_size(s));
  const int64_t b = s->batch, n = s->text_tokens + s->image_tokens;
  const int64_t d = s->heads * 128, hid_w = s->mlp_hidden, mlp_in = flux_mlp_in(s);
  const int64_t big_w = 3 * d + hid_w;
  const float eps = s->eps;
  Carve c{static_cast<unsigned char*>(workspace), 0};
  __nv_bfloat16* nrm = c.take(b * n * d);
  __nv_bfloat16* big = c.take(b * n * big_w);
  __nv_bfloat16* x = static_cast<__nv_bfloat16*>(hidden);
  const __nv_bfloat16* mod = static_cast<const __nv_bfloat16*>(modulation);
  const int64_t bsx = n * d, bsb = n * big_w;
  KINO_TRY(kino_adaln(x, d, bsx, mod, mod + d, bs_modulation, nrm, d, bsx, b, n, d,
                      KINO_NORM_LAYER, eps, stream));
  // [k | v | q | mlp]: k and q normalised and rotated, the MLP activated, in one epilogue
  kino_epilogue e = plain_epi(flux_act_kind(s));
  e.act_col_begin = 3 * d;
  set_qk(&e, w->norm_k, 0, w->norm_q, 2 * d, d, rope, 0, eps);
  KINO_TRY(kino_linear(nrm, w->fused, big, b, n, 3 * d + mlp_in, d, d, bsx, d, big_w, bsb, &e,
                       stream));
  kino_attention_args att = self_attention(b, s->heads, n, big + 2 * d, big, big + d, big + 2 * d,
                                           big_w, bsb);
  KINO_TRY(kino_attention(&att, stream));
  // to_out over the contiguous [attention | act(mlp)] columns
  kino_epilogue eo = plain_epi(kino::EPI_NONE);
  set_gated(&eo, x, d, bsx, mod + 2 * d, bs_modulation);
  return kino_linear(big + 2 * d, w->to_out, x, b, n, d, d + hid_w, big_w, bsb, d + hid_w, d, bsx,
                     &eo, stream);
}

int64_t kino_ltx_video_block_workspace_size(const kino_ltx_block_shape* s) {
  if (s == nullptr || s->batch < 1 || s->tokens < 1 || s->context_tokens < 1 || s->heads < 1 ||
      s->context_dim < 8 || s->ff_hidden < 8) {
    fail(KINO_EINVAL, "kino_ltx_video_block_workspace_size: invalid shape");
    return -1;
  }
  const int64_t b = s->batch, t = s->tokens, tc = s->context_tokens, d = s->heads * 128;
  const int64_t two = 2;
  return align_up(b * t * d * two) + align_up(b * t * s->ff_hidden * two) +
         align_up(b * t * 3 * d * two) + align_up(b * t * s->heads * two) +
         align_up(b * tc * s->context_dim * two) + align_up(b * tc * 2 * d * two);
}

kino_status kino_ltx_video_block(const kino_ltx_block_shape* s,
                                 const kino_ltx_video_block_weights* w, void* hidden,
                                 const void* context, const void* values, int64_t bs_values,
                                 const void* prompt, int64_t bs_prompt, const float* rope_cos,
                                 const float* rope_sin, int rope_batched, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  const int64_t need = kino_ltx_video_block_workspace_size(s);
  if (need < 0) return KINO_EINVAL;
  if (w == nullptr || hidden == nullptr || context == nullptr || values == nullptr ||
      prompt == nullptr || rope_cos == nullptr || rope_sin == nullptr || workspace == nullptr)
    return fail(KINO_EINVAL, "kino_ltx_video_block: null argument");
  if (workspace_bytes < need || !aligned16(workspace))
    return fail(KINO_EINVAL, "kino_ltx_video_block: workspace below %lld bytes or unaligned",
                (long long)need);
  const int64_t b = s->batch, t = s->tokens, tc = s->context_tokens, h = s->heads;
  const int64_t d = h * 128, dc = s->context_dim, ff = s->ff_hidden;
  if (dc != d)
    return fail(KINO_ENOTSUPPORTED,
                "kino_ltx_video_block: the prompt modulation is %lld wide, context width %lld",
                (long long)d, (long long)dc);
  const float eps = s->eps;
  Carve c{static_cast<unsigned char*>(workspace), 0};
  __nv_bfloat16* nrm = c.take(b * t * d);
  __nv_bfloat16* hid = c.take(b * t * ff);
  __nv_bfloat16* qkv = c.take(b * t * 3 * d);
  __nv_bfloat16* gates = c.take(b * t * h);
  __nv_bfloat16* ctxm = c.take(b * tc * dc);
  __nv_bfloat16* ctxkv = c.take(b * tc * 2 * d);
  __nv_bfloat16* x = static_cast<__nv_bfloat16*>(hidden);
  const __nv_bfloat16* val = static_cast<const __nv_bfloat16*>(values);
  const __nv_bfloat16* pr = static_cast<const __nv_bfloat16*>(prompt);
  auto vj = [&](int j) { return val + j * d; };  // (shift, scale, gate) x {attn, ff}, cross q
  const int64_t bsx = t * d, bsq = t * 3 * d, bsg = t * h;
  __nv_bfloat16* vv = qkv;
  __nv_bfloat16* q = qkv + d;
  __nv_bfloat16* k = qkv + 2 * d;
  auto adaln = [&](const __nv_bfloat16* shift, const __nv_bfloat16* scale) {
    return kino_adaln(x, d, bsx, shift, scale, bs_values, nrm, d, bsx, b, t, d, KINO_NORM_RMS,
                      eps, stream);
  };
  auto lin = [&](const void* in, int64_t ldi, int64_t bsi, const void* wt, const void* bias,
                 void* out, int64_t rows, int64_t n_out, int64_t kdim, int64_t ldo, int64_t bso,
                 kino_epilogue e) {
    e.bias = bias;
    return kino_linear(in, wt, out, b, rows, n_out, kdim, ldi, bsi, kdim, ldo, bso, &e, stream);
  };
  // gated self-attention: [v | q | k] projection, full-row q/k norms + split RoPE
  KINO_TRY(adaln(vj(0), vj(1)));
  KINO_TRY(lin(nrm, d, bsx, w->g1_w, w->g1_b, gates, t, h, d, h, bsg, plain_epi(kino::EPI_SIGMOID2)));
  KINO_TRY(lin(nrm, d, bsx, w->qkv_w, w->qkv_b, qkv, t, 3 * d, d, 3 * d, bsq, plain_epi(kino::EPI_NONE)));
  KINO_TRY(kino_qk_norm_rope(q, 3 * d, bsq, b, t, h, w->qn1, KINO_QKNORM_FULL_ROW, KINO_ROPE_SPLIT,
                             rope_cos, rope_sin, rope_batched, t, 0, eps, stream));
  KINO_TRY(kino_qk_norm_rope(k, 3 * d, bsq, b, t, h, w->kn1, KINO_QKNORM_FULL_ROW, KINO_ROPE_SPLIT,
                             rope_cos, rope_sin, rope_batched, t, 0, eps, stream));
  kino_attention_args att = self_attention(b, h, t, q, k, vv, q, 3 * d, bsq);
  att.gate[0] = gates;
  att.ld_gate[0] = h;
  att.bs_gate[0] = bsg;
  KINO_TRY(kino_attention(&att, stream));
  kino_epilogue eg = plain_epi(kino::EPI_NONE);
  set_gated(&eg, x, d, bsx, vj(2), bs_values);
  KINO_TRY(lin(q, 3 * d, bsq, w->o1_w, w->o1_b, x, t, d, d, d, bsx, eg));
  // text cross-attention on the prompt-modulated context
  KINO_TRY(adaln(vj(6), vj(7)));
  KINO_TRY(kino_adaln(context, dc, tc * dc, pr, pr + dc, bs_prompt, ctxm, dc, tc * dc, b, tc, dc,
                      KINO_NORM_NONE, eps, stream));
  KINO_TRY(lin(nrm, d, bsx, w->g2_w, w->g2_b, gates, t, h, d, h, bsg, plain_epi(kino::EPI_SIGMOID2)));
  KINO_TRY(lin(nrm, d, bsx, w->q2_w, w->q2_b, q, t, d, d, 3 * d, bsq, plain_epi(kino::EPI_NONE)));
  KINO_TRY(lin(ctxm, dc, tc * dc, w->kv2_w, w->kv2_b, ctxkv, tc, 2 * d, dc, 2 * d, tc * 2 * d,
               plain_epi(kino::EPI_NONE)));
  KINO_TRY(kino_qk_norm_rope(q, 3 * d, bsq, b, t, h, w->qn2, KINO_QKNORM_FULL_ROW, KINO_ROPE_NONE,
                             nullptr, nullptr, 0, 0, 0, eps, stream));
  KINO_TRY(kino_qk_norm_rope(ctxkv, 2 * d, tc * 2 * d, b, tc, h, w->kn2, KINO_QKNORM_FULL_ROW,
                             KINO_ROPE_NONE, nullptr, nullptr, 0, 0, 0, eps, stream));
  kino_attention_args cross = self_attention(b, h, t, q, ctxkv, ctxkv + d, q, 3 * d, bsq);
  cross.kv_tokens[0] = tc;
  cross.ld_k[0] = cross.ld_v[0] = 2 * d;
  cross.bs_k[0] = cross.bs_v[0] = tc * 2 * d;
  cross.gate[0] = gates;
  cross.ld_gate[0] = h;
  cross.bs_gate[0] = bsg;
  KINO_TRY(kino_attention(&cross, stream));
  set_gated(&eg, x, d, bsx, vj(8), bs_values);
  KINO_TRY(lin(q, 3 * d, bsq, w->o2_w, w->o2_b, x, t, d, d, d, bsx, eg));
  // GELU feed-forward
  KINO_TRY(adaln(vj(3), vj(4)));
  kino_epilogue ea = plain_epi(kino::EPI_GELU);
  KINO_TRY(lin(nrm, d, bsx, w->ff_in_w, w->ff_in_b, hid, t, ff, d, ff, t * ff, ea));
  set_gated(&eg, x, d, bsx, vj(5), bs_values);
  return lin(hid, ff, t * ff, w->ff_out_w, w->ff_out_b, x, t, d, ff, d, bsx, eg);
}

}  // extern "C"

#undef KINO_TRY
