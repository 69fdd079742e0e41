// Whole models: a GGUF file (or image in memory) uploaded to HBM in its own block format, and the one-token step of
// fwd.cu behind the reference's forward-pass interface (c/src/forward.h:113-117: cl_fwd_open, cl_fwd_step, cl_fwd_reset,
// cl_fwd_close). Host code.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "ctx.cuh"
#include "fwd.cuh"
#include "gguf.h"
#include "prefill.cuh"

using namespace clb;

struct clb200_model {
  clb200_ctx *ctx = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  clb200_model_info info{};
  uint8_t *dev = nullptr;          // every tensor, norms / routers as fp32, the key/value cache, the scratch
  size_t dev_bytes = 0;
  FwdArgs args{};
  FwdState *st_host = nullptr;     // pinned mirror of the device state
  int *route_host = nullptr;       // pinned [n_layer * K] sel, then [n_layer * K] weights (as float bits)
  int ctas = 0;
  int pos = 0;
  cudaGraphExec_t gen_graph = nullptr;   // one step that feeds its own choice back (generation)
  // the batched prompt path (clb200_model_prefill)
  std::vector<FwdLayer> hl;        // host copy of the layer table
  std::vector<DevLayer> moe;       // each layer's MoE block as the batched kernels take it
  int pf_cap = 64;                 // tokens per batch: the reference's batch for a model in memory (c/src/forward.c:1048)
  int pf_alloc = 0;                // the batch the buffers below hold
  uint8_t *pf = nullptr;           // device: tokens, X, Q, K, V, rotated Q, attention, Q8_K activations
};

namespace {

struct ArchSpec {
  const char *name;
  int qk_mode, norm_topk, rope_pairs, expert_ff_key, scaled;
};
// the mixture-of-experts rows of the reference's table (c/src/forward.c:41-49)
const ArchSpec ARCHS[] = {
    {"olmoe", 1, 0, 0, 0, 0},
    {"qwen3moe", 2, 1, 0, 1, 0},
    {"qwen3vlmoe", 2, 1, 0, 1, 0},
    {"granitemoe", 0, 1, 1, 0, 1},
};

float half_to_float(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(m | 1024), static_cast<int>(e) - 25);
  return s ? -v : v;
}

// A float copy of a 1-D or 2-D F32 / F16 / BF16 tensor (norm weights, routers).
bool to_floats(const Gguf &g, const GgufTensor &t, std::vector<float> &out) {
  uint64_t n = 1;
  for (uint32_t d = 0; d < t.n_dims; ++d) n *= t.dims[d];
  out.resize(static_cast<size_t>(n));
  const uint8_t *p = g.base + t.offset;
  if (t.type == T_F32) { std::memcpy(out.data(), p, n * 4); return true; }
  if (t.type == T_F16 || t.type == 30) {
    for (uint64_t i = 0; i < n; ++i) {
      uint16_t h;
      std::memcpy(&h, p + 2 * i, 2);
      if (t.type == T_F16) out[i] = half_to_float(h);
      else { const uint32_t b = static_cast<uint32_t>(h) << 16; std::memcpy(&out[i], &b, 4); }
    }
    return true;
  }
  return false;
}

bool kq(uint32_t t) { return t == T_Q4_K || t == T_Q6_K; }

}  // namespace

extern "C" {

static int model_setup(clb200_model *m, const Gguf &g, int n_ctx, char *err, size_t errlen) {
  clb200_ctx *c = m->ctx;
  std::string arch;
  if (!g.get_str("general.architecture", arch)) { errf(err, errlen, "the file names no architecture"); return 1; }
  const ArchSpec *spec = nullptr;
  for (const auto &s : ARCHS) if (arch == s.name) spec = &s;
  if (!spec) { errf(err, errlen, "the device forward pass takes the mixture-of-experts architectures olmoe, qwen3moe, qwen3vlmoe and granitemoe, not \"%s\"", arch.c_str()); return 1; }
  auto U = [&](const char *suffix, uint64_t &v) { return g.get_u64(arch + "." + suffix, v); };
  auto F = [&](const char *suffix, double &v) { return g.get_f64(arch + "." + suffix, v); };
  uint64_t E = 0, H = 0, KVH = 0, FF = 0, ctx_train = 0, NL = 0, NE = 0, K = 0, kl = 0;
  if (!U("embedding_length", E) || !U("attention.head_count", H) || !U("attention.head_count_kv", KVH) ||
      !U(spec->expert_ff_key ? "expert_feed_forward_length" : "feed_forward_length", FF) || !U("context_length", ctx_train) ||
      !U("block_count", NL) || !U("expert_count", NE) || !U("expert_used_count", K)) {
    errf(err, errlen, "the model does not state its hyper-parameters (embedding, heads, expert width, context, layers, experts)");
    return 1;
  }
  double eps = 1e-5, base = 10000.0;
  F("attention.layer_norm_rms_epsilon", eps);
  F("rope.freq_base", base);
  int hd = static_cast<int>(E / std::max<uint64_t>(H, 1));
  if (U("attention.key_length", kl) && kl >= 2 && kl <= 1024 && kl % 2 == 0) hd = static_cast<int>(kl);
  FwdArgs &a = m->args;
  a.E = static_cast<int>(E); a.n_head = static_cast<int>(H); a.n_kv = static_cast<int>(KVH); a.hd = hd;
  a.n_q = a.n_head * hd; a.n_kvw = a.n_kv * hd; a.FF = static_cast<int>(FF); a.NE = static_cast<int>(NE); a.K = static_cast<int>(K);
  a.n_layer = static_cast<int>(NL);
  a.qk_mode = spec->qk_mode; a.norm_topk = spec->norm_topk; a.rope_pairs = spec->rope_pairs;
  a.eps = static_cast<float>(eps); a.rope_base = static_cast<float>(base);
  a.embed_scale = a.resid_scale = a.logit_scale = 1.0f; a.attn_scale = 0.f;
  if (spec->scaled) {
    double v;
    if (F("embedding_scale", v)) a.embed_scale = static_cast<float>(v);
    if (F("residual_scale", v)) a.resid_scale = static_cast<float>(v);
    if (F("logit_scale", v) && v > 0) a.logit_scale = static_cast<float>(v);
    if (F("attention.scale", v) && v > 0) a.attn_scale = static_cast<float>(v);
  }
  if (a.attn_scale <= 0) a.attn_scale = 1.0f / std::sqrt(static_cast<float>(hd));
  uint64_t rd = 0;
  if (U("rope.dimension_count", rd) && static_cast<int>(rd) != hd) { errf(err, errlen, "partial rotary embeddings are not implemented"); return 1; }
  if (a.E < 256 || a.E % 256 || a.E > 4096 || a.FF % 256 || a.FF < 256 || a.FF > 4096 || a.n_q % 256 || a.n_q > 4096 ||
      a.n_head < 1 || a.n_kv < 1 || a.n_head % a.n_kv || a.n_head / a.n_kv > FWD_MAX_GROUP || (hd != 64 && hd != 128 && hd != 256) ||
      a.NE < 1 || a.NE > FWD_MAX_NE || a.K < 1 || a.K > FWD_MAX_K || a.K > a.NE || a.n_layer < 1) {
    errf(err, errlen, "shape outside what the device step takes (embedding %d, heads %d/%d x %d, expert width %d, experts %d, used %d)",
         a.E, a.n_head, a.n_kv, hd, a.FF, a.NE, a.K);
    return 1;
  }
  if (spec->qk_mode != 2 && a.n_q != a.E) { errf(err, errlen, "head_dim * heads must equal the embedding width for this architecture"); return 1; }
  a.ctx = n_ctx > 0 ? std::min<int>(n_ctx, static_cast<int>(ctx_train)) : std::min<int>(512, static_cast<int>(ctx_train));

  // ---- tensors: check, then lay out one device block ----------------------------------------------------------------
  struct Item { const GgufTensor *t; size_t off; bool as_float; std::vector<float> f; };
  std::vector<Item> items;
  size_t total = 0;
  auto add = [&](const GgufTensor *t, bool as_float) -> size_t {
    Item it{t, 0, as_float, {}};
    if (as_float && !to_floats(g, *t, it.f)) return SIZE_MAX;
    total = al(total, 256);
    it.off = total;
    total += as_float ? it.f.size() * 4 : t->nbytes;
    total += 64;   // slack: block readers load whole aligned words
    items.push_back(std::move(it));
    return items.back().off;
  };
  auto need = [&](const std::string &name, int dims, uint64_t d0, uint64_t d1, uint64_t d2) -> const GgufTensor * {
    const GgufTensor *t = g.find(name);
    if (!t) { errf(err, errlen, "missing tensor %s", name.c_str()); return nullptr; }
    if (static_cast<int>(t->n_dims) < dims || t->dims[0] != d0 || (dims > 1 && t->dims[1] != d1) || (dims > 2 && t->dims[2] != d2)) {
      errf(err, errlen, "tensor %s has the wrong shape", name.c_str());
      return nullptr;
    }
    return t;
  };
  const GgufTensor *emb = g.find("token_embd.weight");
  if (!emb || emb->n_dims < 2 || emb->dims[0] != E) { errf(err, errlen, "token_embd.weight is missing or not [%d, vocab]", a.E); return 1; }
  a.vocab = static_cast<int>(emb->dims[1]);
  if (emb->type != T_Q4_K && emb->type != T_Q6_K && emb->type != T_Q8_0 && emb->type != T_F32) { errf(err, errlen, "token_embd.weight is %s", type_name(emb->type)); return 1; }
  const GgufTensor *out = g.find("output.weight");
  if (!out) out = emb;   // tied embeddings (c/src/forward.c:186-187)
  if (out->dims[0] != E || out->dims[1] != static_cast<uint64_t>(a.vocab) || !kq(out->type)) { errf(err, errlen, "output.weight must be a Q4_K or Q6_K [%d, %d] matrix", a.E, a.vocab); return 1; }
  const GgufTensor *onorm = need("output_norm.weight", 1, E, 0, 0);
  if (!onorm) return 1;
  const size_t o_emb = add(emb, false), o_out = out == emb ? o_emb : add(out, false), o_onorm = add(onorm, true);
  if (o_onorm == SIZE_MAX) { errf(err, errlen, "output_norm.weight is not a float tensor"); return 1; }
  struct LayerOffs { size_t an, fn, qn, kn, router, wq, wk, wv, wo, gate, up, down; const GgufTensor *t[7]; };
  std::vector<LayerOffs> lo(static_cast<size_t>(a.n_layer));
  const int QN = spec->qk_mode == 2 ? hd : a.n_q, KN = spec->qk_mode == 2 ? hd : a.n_kvw;
  for (int l = 0; l < a.n_layer; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const GgufTensor *an = need(p + "attn_norm.weight", 1, E, 0, 0), *fn = need(p + "ffn_norm.weight", 1, E, 0, 0);
    const GgufTensor *wq = need(p + "attn_q.weight", 2, E, a.n_q, 0), *wk = need(p + "attn_k.weight", 2, E, a.n_kvw, 0);
    const GgufTensor *wv = need(p + "attn_v.weight", 2, E, a.n_kvw, 0), *wo = need(p + "attn_output.weight", 2, a.n_q, E, 0);
    const GgufTensor *rt = need(p + "ffn_gate_inp.weight", 2, E, NE, 0);
    const GgufTensor *ge = need(p + "ffn_gate_exps.weight", 3, E, FF, NE), *ue = need(p + "ffn_up_exps.weight", 3, E, FF, NE);
    const GgufTensor *de = need(p + "ffn_down_exps.weight", 3, FF, E, NE);
    if (!an || !fn || !wq || !wk || !wv || !wo || !rt || !ge || !ue || !de) return 1;
    const GgufTensor *qn = nullptr, *kn = nullptr;
    if (spec->qk_mode) {
      qn = need(p + "attn_q_norm.weight", 1, QN, 0, 0);
      kn = need(p + "attn_k_norm.weight", 1, KN, 0, 0);
      if (!qn || !kn) return 1;
    }
    if (!kq(wq->type) || !kq(wk->type) || !kq(wv->type) || !kq(wo->type)) { errf(err, errlen, "layer %d: the attention matrices must be Q4_K or Q6_K", l); return 1; }
    if (!kq(ge->type) || ge->type != ue->type || !kq(de->type)) { errf(err, errlen, "layer %d: experts must be Q4_K or Q6_K (gate and up alike)", l); return 1; }
    LayerOffs &o = lo[static_cast<size_t>(l)];
    o.an = add(an, true); o.fn = add(fn, true); o.router = add(rt, true);
    o.qn = qn ? add(qn, true) : 0; o.kn = kn ? add(kn, true) : 0;
    if (o.an == SIZE_MAX || o.fn == SIZE_MAX || o.router == SIZE_MAX || o.qn == SIZE_MAX || o.kn == SIZE_MAX) { errf(err, errlen, "layer %d: a norm or router tensor is not float", l); return 1; }
    o.wq = add(wq, false); o.wk = add(wk, false); o.wv = add(wv, false); o.wo = add(wo, false);
    o.gate = add(ge, false); o.up = add(ue, false); o.down = add(de, false);
    o.t[0] = wq; o.t[1] = wk; o.t[2] = wv; o.t[3] = wo; o.t[4] = ge; o.t[5] = ue; o.t[6] = de;
  }
  // key/value cache and scratch
  const size_t kv_elems = static_cast<size_t>(a.n_layer) * a.ctx * a.n_kvw;
  auto take = [&](size_t bytes) { total = al(total, 256); const size_t at = total; total += bytes + 64; return at; };
  const size_t o_kc = take(kv_elems * 2), o_vc = take(kv_elems * 2);
  const size_t o_x = take(a.E * 4), o_qkv = take((a.n_q + 2 * a.n_kvw) * 4), o_att = take(a.n_q * 4);
  const size_t o_rl = take(a.NE * 4), o_hg = take(static_cast<size_t>(a.K) * a.FF * 4), o_lg = take(static_cast<size_t>(a.vocab) * 4);
  const size_t o_rs = take(static_cast<size_t>(a.n_layer) * a.K * 4), o_rw = take(static_cast<size_t>(a.n_layer) * a.K * 4);
  const size_t o_gen = take(static_cast<size_t>(a.ctx) * 4), o_layers = take(sizeof(FwdLayer) * a.n_layer), o_st = take(sizeof(FwdState));
  const size_t o_rope = take(static_cast<size_t>(a.ctx) * hd * 4);

  // ---- the shared-memory plan -------------------------------------------------------------------------------------------
  const int G = c->sms, NW = FWD_THREADS / 32;
  const int nb = a.E / 256, nbd = a.FF / 256;
  a.rgu_max = (a.FF + G - 1) / G;
  a.rd_max = (a.E + G - 1) / G;
  a.nre_max = (a.NE + G - 1) / G;
  uint32_t gt = lo[0].t[4]->type, dt = lo[0].t[6]->type;
  for (int l = 1; l < a.n_layer; ++l)
    if (lo[static_cast<size_t>(l)].t[4]->type != gt || lo[static_cast<size_t>(l)].t[6]->type != dt) { gt = 0; break; }
  // rows of any layer's experts: size the slots for the wider of the two types
  a.grb = static_cast<uint32_t>(row_bytes(T_Q6_K, a.E));
  a.drb = static_cast<uint32_t>(row_bytes(T_Q6_K, a.FF));
  if (gt == T_Q4_K) a.grb = static_cast<uint32_t>(row_bytes(T_Q4_K, a.E));
  if (gt != 0 && dt == T_Q4_K) a.drb = static_cast<uint32_t>(row_bytes(T_Q4_K, a.FF));
  a.gseg = static_cast<uint32_t>(al(static_cast<size_t>(a.rgu_max) * a.grb + 32, 16));
  a.slot_bytes = 2 * a.gseg;
  a.dslot_bytes = static_cast<uint32_t>(al(static_cast<size_t>(a.rd_max) * a.drb + 32, 16));
  const int XQW = std::max(a.E, a.n_q);
  size_t o = 0;
  auto st_take = [&](size_t bytes, size_t align = 16) { const size_t at = al(o, align); o = at + bytes; return static_cast<uint32_t>(at); };
  a.off_bars = st_take(8 * (a.K + 3 + HEAD_STAGES));
  a.off_xn = st_take(static_cast<size_t>(a.E) * 4);
  a.off_xq = st_take(XQW + 2 * (XQW / 16) + 4 * (XQW / 256));
  a.off_misc = st_take(NW * 8 + 8 * 4 + 3 * 32 * 4 + FWD_MAX_NE * 4 + NW * 8 + FWD_MAX_NE * 4 + 4 * 32 * 4);
  a.off_router = st_take(static_cast<size_t>(a.nre_max) * a.E * 4);
  // the router products, then each row's weighted expert outputs [rd_max][K]
  a.off_rprod = st_take(std::max<size_t>(static_cast<size_t>(a.nre_max) * 8 * (a.E / 8 + 4), static_cast<size_t>(a.rd_max) * a.K) * 4);
  a.off_terms = st_take(std::max<size_t>(static_cast<size_t>(a.rd_max) * a.K * nbd * 4, 2 * NW * 8));
  a.off_hq = st_take(static_cast<size_t>(a.K) * a.FF + 2 * (static_cast<size_t>(a.K) * a.FF / 16) + 4 * (static_cast<size_t>(a.K) * a.FF / 256));
  a.off_xr = st_take(static_cast<size_t>(a.rd_max) * 4);
  // the slots hold a layer's dense rows (each CTA's rows of wq, wk, wv, wo, one segment after another: fwd.cu's
  // dense_offset) and then the chosen experts' gate/up rows
  size_t dense_need = 0;
  {
    uint64_t rbmax[4] = {0, 0, 0, 0};
    for (int l = 0; l < a.n_layer; ++l)
      for (int q = 0; q < 4; ++q) rbmax[q] = std::max<uint64_t>(rbmax[q], gguf_row_bytes(lo[static_cast<size_t>(l)].t[q]->type, lo[static_cast<size_t>(l)].t[q]->dims[0]));
    const int QKVR = a.n_q + 2 * a.n_kvw;
    for (int cc = 0; cc < G; ++cc) {
      const int q0 = static_cast<int>(static_cast<int64_t>(QKVR) * cc / G), q1 = static_cast<int>(static_cast<int64_t>(QKVR) * (cc + 1) / G);
      const int e0 = static_cast<int>(static_cast<int64_t>(a.E) * cc / G), e1 = static_cast<int>(static_cast<int64_t>(a.E) * (cc + 1) / G);
      const int cnt[4] = {std::max(0, std::min(q1, a.n_q) - std::max(q0, 0)),
                          std::max(0, std::min(q1 - a.n_q, a.n_kvw) - std::max(q0 - a.n_q, 0)),
                          std::max(0, std::min(q1 - a.n_q - a.n_kvw, a.n_kvw) - std::max(q0 - a.n_q - a.n_kvw, 0)), e1 - e0};
      size_t need = 0;
      for (int q = 0; q < 4; ++q) need += al(static_cast<size_t>(cnt[q]) * rbmax[q] + 32, 16);
      dense_need = std::max(dense_need, need);
    }
  }
  const size_t slots_size = al(std::max<size_t>(static_cast<size_t>(a.K) * a.slot_bytes, dense_need), 128);
  a.off_slots = st_take(slots_size, 128);
  // the dslots, right after the slots, hold the chosen experts' down rows, or the attention scratch of a query head: its
  // query, rotary row and QK-norm weights [hd] floats each, the new key and value [hd] halves each, FWD_ATT_BLOCK staged
  // key or value rows, the scores of every position, and per 256-position chunk its maximum, sum and [hd] value sums; the
  // output matrix's stages span both regions
  const int grp = a.n_head / a.n_kv;
  const bool can_group = grp >= 2 && grp <= FWD_MAX_GROUP;   // else every step takes the plain path over the whole context
  const size_t att_chunks = can_group ? (static_cast<size_t>(a.ctx) + FWD_ATT_CHUNK - 1) / FWD_ATT_CHUNK : 1;
  const size_t att_scores = can_group ? FWD_ATT_CHUNK : (static_cast<size_t>(a.ctx) + 3) & ~size_t(3);
  const size_t att_need = static_cast<size_t>(hd) * 20 + static_cast<size_t>(FWD_ATT_BLOCK) * (hd + 8) * 2 + att_scores * 4 +
                          att_chunks * (2 + hd) * 4;
  const size_t head_need = static_cast<size_t>(HEAD_STAGES) * al(HEAD_ROWS * row_bytes(out->type, a.E) + 32, 16);
  const size_t dslots_size = std::max<size_t>(std::max<size_t>(static_cast<size_t>(a.K) * a.dslot_bytes, att_need),
                                              head_need > slots_size ? head_need - slots_size : 0);
  a.off_dslots = st_take(dslots_size, 128);
  if (a.off_dslots != a.off_slots + slots_size) { errf(err, errlen, "internal: the slots and dslots are not adjacent"); return 1; }
  a.smem_bytes = static_cast<uint32_t>(o + 16);
  (void)nb;
  if (a.smem_bytes > static_cast<uint32_t>(c->max_smem)) {
    errf(err, errlen, "the step needs %u bytes of shared memory per CTA, the device gives %d", a.smem_bytes, c->max_smem);
    return 1;
  }

  // ---- upload ------------------------------------------------------------------------------------------------------------
  cudaSetDevice(c->device);
  CUDA_OR(cudaMalloc(&m->dev, total), "allocating the model in HBM");
  m->dev_bytes = total;
  CUDA_OR(cudaMemset(m->dev, 0, total), "clearing the model block");
  for (const Item &it : items) {
    const void *src = it.as_float ? static_cast<const void *>(it.f.data()) : static_cast<const void *>(g.base + it.t->offset);
    const size_t n = it.as_float ? it.f.size() * 4 : it.t->nbytes;
    CUDA_OR(cudaMemcpy(m->dev + it.off, src, n, cudaMemcpyHostToDevice), "uploading a tensor");
  }
  auto mat = [&](size_t off, const GgufTensor *t) { return FwdMat{m->dev + off, t->type, static_cast<uint32_t>(gguf_row_bytes(t->type, t->dims[0]))}; };
  std::vector<FwdLayer> layers(static_cast<size_t>(a.n_layer));
  for (int l = 0; l < a.n_layer; ++l) {
    const LayerOffs &q = lo[static_cast<size_t>(l)];
    FwdLayer &y = layers[static_cast<size_t>(l)];
    y.attn_norm = reinterpret_cast<const float *>(m->dev + q.an);
    y.ffn_norm = reinterpret_cast<const float *>(m->dev + q.fn);
    y.qn = spec->qk_mode ? reinterpret_cast<const float *>(m->dev + q.qn) : nullptr;
    y.kn = spec->qk_mode ? reinterpret_cast<const float *>(m->dev + q.kn) : nullptr;
    y.router = reinterpret_cast<const float *>(m->dev + q.router);
    y.wq = mat(q.wq, q.t[0]); y.wk = mat(q.wk, q.t[1]); y.wv = mat(q.wv, q.t[2]); y.wo = mat(q.wo, q.t[3]);
    y.gate = m->dev + q.gate; y.up = m->dev + q.up; y.down = m->dev + q.down;
    y.gate_type = q.t[4]->type; y.down_type = q.t[6]->type;
    y.gate_slab = row_bytes(y.gate_type, a.E) * a.FF;
    y.up_slab = y.gate_slab;
    y.down_slab = row_bytes(y.down_type, a.FF) * a.E;
    if (row_bytes(y.gate_type, a.E) > a.grb || row_bytes(y.down_type, a.FF) > a.drb) { errf(err, errlen, "layer %d: expert row wider than planned", l); return 1; }
  }
  CUDA_OR(cudaMemcpy(m->dev + o_layers, layers.data(), sizeof(FwdLayer) * layers.size(), cudaMemcpyHostToDevice), "uploading the layer table");
  m->hl = layers;
  m->moe.resize(layers.size());
  for (size_t l = 0; l < layers.size(); ++l) {   // the MoE block of each layer for the batched kernels (device pointers)
    const FwdLayer &y = layers[l];
    clb200_moe_layer &d = m->moe[l].d;
    d.ffn_norm_f = y.ffn_norm;
    d.router_f = y.router;
    d.gate = clb200_w{y.gate, y.gate_type, a.FF, a.E};
    d.up = clb200_w{y.up, y.gate_type, a.FF, a.E};
    d.down = clb200_w{y.down, y.down_type, a.E, a.FF};
    d.gate_slab = y.gate_slab;
    d.up_slab = y.up_slab;
    d.down_slab = y.down_slab;
    d.n_embd = a.E;
    d.n_ff_exp = a.FF;
    d.n_expert = a.NE;
    d.n_used = a.K;
    d.norm_topk = a.norm_topk;
    d.resid_scale = a.resid_scale;
    d.rms_eps = a.eps;
    m->moe[l].live = true;
  }
  a.tok_embd = mat(o_emb, emb);
  a.output = mat(o_out, out);
  a.out_norm = reinterpret_cast<const float *>(m->dev + o_onorm);
  a.layers = reinterpret_cast<const FwdLayer *>(m->dev + o_layers);
  a.kc = reinterpret_cast<__half *>(m->dev + o_kc);
  a.vc = reinterpret_cast<__half *>(m->dev + o_vc);
  a.x = reinterpret_cast<float *>(m->dev + o_x);
  a.qkv = reinterpret_cast<float *>(m->dev + o_qkv);
  a.att = reinterpret_cast<float *>(m->dev + o_att);
  {   // the rotary angles' cosines and sines exactly as the reference computes them (c/src/forward.c:420-435): the same
      // float expression and the same C library's powf, cosf and sinf, for every position of the context
    const int H = hd / 2;
    std::vector<float> freq(static_cast<size_t>(H)), cs(static_cast<size_t>(a.ctx) * hd);
    for (int i = 0; i < H; ++i) freq[static_cast<size_t>(i)] = powf(a.rope_base, -2.0f * static_cast<float>(i) / static_cast<float>(hd));
    for (int p = 0; p < a.ctx; ++p)
      for (int i = 0; i < H; ++i) {
        const float theta = static_cast<float>(p) * freq[static_cast<size_t>(i)];
        cs[static_cast<size_t>(p) * hd + i] = cosf(theta);
        cs[static_cast<size_t>(p) * hd + H + i] = sinf(theta);
      }
    CUDA_OR(cudaMemcpy(m->dev + o_rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "uploading the rotary tables");
    a.rope_cs = reinterpret_cast<const float *>(m->dev + o_rope);
  }
  a.rlogits = reinterpret_cast<float *>(m->dev + o_rl);
  a.hg = reinterpret_cast<float *>(m->dev + o_hg);
  a.logits = reinterpret_cast<float *>(m->dev + o_lg);
  a.route_sel = reinterpret_cast<int *>(m->dev + o_rs);
  a.route_wt = reinterpret_cast<float *>(m->dev + o_rw);
  a.gen_out = reinterpret_cast<int *>(m->dev + o_gen);
  a.st = reinterpret_cast<FwdState *>(m->dev + o_st);
  a.trace = nullptr;
  a.feed = 0;
  CUDA_OR(fwd_allow_smem(c->max_smem), "kernel attribute");
  CUDA_OR(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "creating a stream");
  CUDA_OR(cudaMallocHost(&m->st_host, sizeof(FwdState)), "pinned state");
  CUDA_OR(cudaMallocHost(&m->route_host, static_cast<size_t>(a.n_layer) * a.K * 8), "pinned routing");
  m->ctas = G;
  clb200_model_info &in = m->info;
  std::snprintf(in.arch, sizeof in.arch, "%s", arch.c_str());
  in.n_layer = a.n_layer; in.n_embd = a.E; in.n_head = a.n_head; in.n_head_kv = a.n_kv; in.head_dim = hd;
  in.n_ff_exp = a.FF; in.n_expert = a.NE; in.n_used = a.K; in.n_vocab = a.vocab; in.n_ctx = a.ctx;
  in.device_bytes = total;
  in.smem_bytes = a.smem_bytes;
  return 0;
}

clb200_model *clb200_model_open_image(clb200_ctx *c, const void *image, size_t bytes, int n_ctx, char *err, size_t errlen) {
  if (!c || !image) { errf(err, errlen, "no context or image"); return nullptr; }
  Gguf g;
  if (g.parse(static_cast<const uint8_t *>(image), bytes, err, errlen)) return nullptr;
  auto *m = new clb200_model();
  m->ctx = c;
  m->device = c->device;
  if (model_setup(m, g, n_ctx, err, errlen)) { clb200_model_close(m); return nullptr; }
  return m;
}

clb200_model *clb200_model_open(clb200_ctx *c, const char *path, int n_ctx, char *err, size_t errlen) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) { errf(err, errlen, "cannot open %s", path); return nullptr; }
  struct stat sb{};
  if (fstat(fd, &sb) || sb.st_size <= 0) { ::close(fd); errf(err, errlen, "cannot read %s", path); return nullptr; }
  void *map = mmap(nullptr, static_cast<size_t>(sb.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED) { errf(err, errlen, "cannot map %s", path); return nullptr; }
  clb200_model *m = clb200_model_open_image(c, map, static_cast<size_t>(sb.st_size), n_ctx, err, errlen);
  munmap(map, static_cast<size_t>(sb.st_size));   // everything the step reads is in HBM now
  return m;
}

void clb200_model_close(clb200_model *m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  if (m->gen_graph) cudaGraphExecDestroy(m->gen_graph);
  if (m->dev) cudaFree(m->dev);
  if (m->st_host) cudaFreeHost(m->st_host);
  if (m->route_host) cudaFreeHost(m->route_host);
  if (m->pf) cudaFree(m->pf);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

int clb200_model_get_info(const clb200_model *m, clb200_model_info *out) {
  if (!m || !out) return 1;
  *out = m->info;
  return 0;
}

void clb200_model_reset(clb200_model *m) {
  if (m) m->pos = 0;
}

int clb200_model_pos(const clb200_model *m) { return m ? m->pos : -1; }

static const char *fwd_error_text(int code) {
  switch (code) {
    case ERR_WAIT_ROUTER: return "timed out waiting for the router logits of other CTAs";
    case ERR_WAIT_COPY: return "timed out waiting for a bulk copy into shared memory";
    case ERR_BAD_EXPERT: return "token or position out of range";
    case ERR_WAIT_GRID: return "timed out at a grid barrier (are all CTAs resident?)";
    default: return "unknown device error";
  }
}

// Writes (token, pos) into the device state and launches one step; asynchronous on the model's stream.
static int launch_step(clb200_model *m, int token, int feed, char *err, size_t errlen) {
  FwdState s{};
  s.token = token;
  s.pos = m->pos;
  *m->st_host = s;
  CUDA_OR(cudaMemcpyAsync(m->args.st, m->st_host, sizeof(FwdState), cudaMemcpyHostToDevice, m->stream), "state upload");
  FwdArgs a = m->args;
  a.feed = feed;
  a.trace = m->ctx->trace;
  a.force_miss = m->ctx->force_miss;
  CUDA_OR(fwd_launch(a, m->ctas, m->stream), "launching the step");
  return 0;
}

int clb200_model_step(clb200_model *m, int token, float *logits, int *next_token, int *sel_out, float *wt_out, char *err,
                      size_t errlen) {
  if (!m) { errf(err, errlen, "no model"); return 1; }
  const FwdArgs &a = m->args;
  if (token < 0 || token >= a.vocab) { errf(err, errlen, "token %d is outside the vocabulary", token); return 1; }
  if (m->pos >= a.ctx) { errf(err, errlen, "the context is full (%d tokens)", a.ctx); return 1; }
  cudaSetDevice(m->device);
  if (launch_step(m, token, 0, err, errlen)) return 1;
  CUDA_OR(cudaMemcpyAsync(m->st_host, a.st, sizeof(FwdState), cudaMemcpyDeviceToHost, m->stream), "state download");
  const size_t nr = static_cast<size_t>(a.n_layer) * a.K;
  if (sel_out || wt_out) {
    CUDA_OR(cudaMemcpyAsync(m->route_host, a.route_sel, nr * 4, cudaMemcpyDeviceToHost, m->stream), "routing download");
    CUDA_OR(cudaMemcpyAsync(m->route_host + nr, a.route_wt, nr * 4, cudaMemcpyDeviceToHost, m->stream), "routing download");
  }
  if (logits) CUDA_OR(cudaMemcpyAsync(logits, a.logits, static_cast<size_t>(a.vocab) * 4, cudaMemcpyDeviceToHost, m->stream), "logits download");
  CUDA_OR(cudaStreamSynchronize(m->stream), "running the step");
  if (m->st_host->err) { errf(err, errlen, "device error %d: %s", m->st_host->err, fwd_error_text(m->st_host->err)); return 1; }
  if (sel_out) std::memcpy(sel_out, m->route_host, nr * 4);
  if (wt_out) std::memcpy(wt_out, m->route_host + nr, nr * 4);
  if (next_token) *next_token = m->st_host->next;
  m->pos++;
  return 0;
}

int clb200_model_generate(clb200_model *m, int token, int n, int *tokens_out, char *err, size_t errlen) {
  if (!m) { errf(err, errlen, "no model"); return 1; }
  const FwdArgs &a = m->args;
  if (n < 1) return 0;
  if (token < 0 || token >= a.vocab) { errf(err, errlen, "token %d is outside the vocabulary", token); return 1; }
  if (m->pos + n > a.ctx) { errf(err, errlen, "%d more tokens do not fit the context (%d of %d used)", n, m->pos, a.ctx); return 1; }
  cudaSetDevice(m->device);
  const int start = m->pos;
  if (!m->gen_graph) {   // one step that feeds its own choice back, captured once, replayed n times
    FwdArgs g = a;
    g.feed = 1;
    g.trace = nullptr;
    g.force_miss = m->ctx->force_miss;   // as the graph is captured
    cudaGraph_t graph = nullptr;
    CUDA_OR(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "capturing the step");
    const cudaError_t le = fwd_launch(g, m->ctas, m->stream);
    const cudaError_t ce = cudaStreamEndCapture(m->stream, &graph);
    if (le != cudaSuccess || ce != cudaSuccess) { errf(err, errlen, "capturing the step: %s", cudaGetErrorString(le != cudaSuccess ? le : ce)); if (graph) cudaGraphDestroy(graph); return 1; }
    const cudaError_t ie = cudaGraphInstantiate(&m->gen_graph, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) { errf(err, errlen, "instantiating the step graph: %s", cudaGetErrorString(ie)); m->gen_graph = nullptr; return 1; }
  }
  FwdState s{};
  s.token = token;
  s.pos = start;
  *m->st_host = s;
  CUDA_OR(cudaMemcpyAsync(a.st, m->st_host, sizeof(FwdState), cudaMemcpyHostToDevice, m->stream), "state upload");
  for (int i = 0; i < n; ++i) CUDA_OR(cudaGraphLaunch(m->gen_graph, m->stream), "replaying the step");
  CUDA_OR(cudaMemcpyAsync(m->st_host, a.st, sizeof(FwdState), cudaMemcpyDeviceToHost, m->stream), "state download");
  if (tokens_out) CUDA_OR(cudaMemcpyAsync(tokens_out, a.gen_out + start, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, m->stream), "tokens download");
  CUDA_OR(cudaStreamSynchronize(m->stream), "generating");
  if (m->st_host->err) { errf(err, errlen, "device error %d: %s", m->st_host->err, fwd_error_text(m->st_host->err)); return 1; }
  m->pos = start + n;
  return 0;
}

int clb200_model_generate_async(clb200_model *m, int token, int n, void *stream, char *err, size_t errlen) {
  // the same replay on a caller's stream with no host synchronisation (for timing); tokens via clb200_model_tokens
  if (!m) { errf(err, errlen, "no model"); return 1; }
  const FwdArgs &a = m->args;
  if (m->pos + n > a.ctx || n < 1 || !m->gen_graph) { errf(err, errlen, "generate once synchronously first, and stay inside the context"); return 1; }
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  FwdState s{};
  s.token = token;
  s.pos = m->pos;
  *m->st_host = s;
  CUDA_OR(cudaMemcpyAsync(a.st, m->st_host, sizeof(FwdState), cudaMemcpyHostToDevice, st), "state upload");
  for (int i = 0; i < n; ++i) CUDA_OR(cudaGraphLaunch(m->gen_graph, st), "replaying the step");
  m->pos += n;
  return 0;
}

int clb200_model_tokens(clb200_model *m, int start, int n, int *tokens_out, char *err, size_t errlen) {
  if (!m || start < 0 || n < 0 || start + n > m->args.ctx) { errf(err, errlen, "range outside the context"); return 1; }
  CUDA_OR(cudaMemcpy(tokens_out, m->args.gen_out + start, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost), "tokens download");
  CUDA_OR(cudaMemcpy(m->st_host, m->args.st, sizeof(FwdState), cudaMemcpyDeviceToHost), "state download");
  if (m->st_host->err) { errf(err, errlen, "device error %d: %s", m->st_host->err, fwd_error_text(m->st_host->err)); return 1; }
  return 0;
}

// ---- the batched prompt path: the reference's cl_fwd_prefill / run_std (c/src/forward.c:1078-1225, 1256-1282) ----------

// Buffers of the batched path for batches of up to `cap` tokens, carved from one device block.
struct PfBufs {
  int *tok;
  float *X, *Q, *K, *V, *Qr, *att;
  int8_t *qs;
  float *dd;
  int16_t *bs;
  PfTc tc;
  size_t total;
};
static PfBufs pf_layout(const FwdArgs &a, int cap, uint8_t *base) {
  PfBufs b{};
  size_t o = 0;
  auto take = [&](size_t n) { const size_t at = o; o += (n + 255) & ~size_t(255); return base + at; };
  const size_t C = static_cast<size_t>(cap), W = static_cast<size_t>(std::max(a.E, a.n_q));
  b.tok = reinterpret_cast<int *>(take(C * 4));
  b.X = reinterpret_cast<float *>(take(C * a.E * 4));
  b.Q = reinterpret_cast<float *>(take(C * a.n_q * 4));
  b.K = reinterpret_cast<float *>(take(C * a.n_kvw * 4));
  b.V = reinterpret_cast<float *>(take(C * a.n_kvw * 4));
  b.Qr = reinterpret_cast<float *>(take(C * a.n_q * 4));
  b.att = reinterpret_cast<float *>(take(C * a.n_q * 4));
  b.qs = reinterpret_cast<int8_t *>(take(C * W));
  b.dd = reinterpret_cast<float *>(take(C * W / 256 * 4));
  b.bs = reinterpret_cast<int16_t *>(take(C * W / 16 * 2));
  b.tc.co = reinterpret_cast<int *>(take(16));
  b.tc.ph = reinterpret_cast<__half *>(take(C * W * 2));
  b.tc.pl = reinterpret_cast<__half *>(take(C * W * 2));
  b.tc.rs = reinterpret_cast<float *>(take(C * 4));
  b.tc.tmp = reinterpret_cast<float *>(take(C * W * 4));
  b.total = o;
  return b;
}

#define PF_OR(call, msg)                                                                                              \
  do {                                                                                                                \
    const int e_ = static_cast<int>(call);                                                                            \
    if (e_) { errf(err, errlen, "%s: %s", msg, cudaGetErrorString(static_cast<cudaError_t>(e_))); return 1; }         \
  } while (0)

// nb tokens (2 <= nb <= the batch) at positions pos .. pos + nb - 1 through every layer together; the logits after the last
// one into `logits` (host) when it is not null.
static int prefill_batch(clb200_model *m, const int *tokens, int nb, float *logits, char *err, size_t errlen) {
  const FwdArgs &a = m->args;
  const int E = a.E, NQ = a.n_q, KW = a.n_kvw, pos0 = m->pos;
  const cudaStream_t st = m->stream;
  const PfBufs b = pf_layout(a, m->pf_alloc, m->pf);
  int *errw = m->ctx->small;
  CUDA_OR(cudaMemcpyAsync(b.tok, tokens, static_cast<size_t>(nb) * 4, cudaMemcpyHostToDevice, st), "tokens upload");
  PF_OR(pf_embed(a.tok_embd, b.tok, nb, E, a.embed_scale, b.X, st), "the embedding");
  for (int l = 0; l < a.n_layer; ++l) {
    const FwdLayer &y = m->hl[static_cast<size_t>(l)];
    __half *kc = a.kc + static_cast<size_t>(l) * a.ctx * KW, *vc = a.vc + static_cast<size_t>(l) * a.ctx * KW;
    // attention (c/src/forward.c:1096-1123): norm, Q/K/V products, QK-norm + rotation + cache, attention, O product
    PF_OR(pf_norm_q8k(b.X, 0, nb, E, y.attn_norm, a.eps, b.qs, b.dd, b.bs, st), "the attention norm");
    // the dense products: Q4_K on the tensor cores unless the integer path is asked for (clb200_set_exact)
    const bool tc = !m->ctx->exact;
    auto dense = [&](const FwdMat &w, int rows, int cols, float *out, int accum, float scale) {
      return tc ? pf_mv_tc(w, rows, cols, nb, b.qs, b.dd, b.bs, out, accum, scale, b.tc, errw, st)
                : pf_mv(w, rows, cols, nb, b.qs, b.dd, b.bs, out, accum, scale, errw, st);
    };
    PF_OR(dense(y.wq, NQ, E, b.Q, 0, 1.f), "the Q product");
    PF_OR(dense(y.wk, KW, E, b.K, 0, 1.f), "the K product");
    PF_OR(dense(y.wv, KW, E, b.V, 0, 1.f), "the V product");
    PfQkArgs qa{b.Q, b.K, b.V, b.Qr, y.qn, y.kn, kc, vc, a.rope_cs, nb, pos0, a.n_head, a.n_kv, a.hd, a.qk_mode, a.rope_pairs, a.eps};
    PF_OR(pf_qk(qa, st), "QK-norm and rotation");
    PfAttnArgs aa{b.Qr, kc, vc, b.att, nb, pos0, a.n_head, a.n_kv, a.hd, KW, a.attn_scale};
    PF_OR(pf_attn(aa, st), "the attention");
    PF_OR(pf_q8k(b.att, nb, NQ, b.qs, b.dd, b.bs, st), "quantizing the attention");
    PF_OR(dense(y.wo, E, NQ, b.X, 1, a.resid_scale), "the O product");
    // the mixture of experts over the batch (c/src/forward.c:1131-1210): the batched kernels
    if (run_moe_block(m->ctx, m->moe[static_cast<size_t>(l)], b.X, nb, nullptr, nullptr, st, err, errlen)) return 1;
  }
  if (logits) {   // the distribution after the last token (c/src/forward.c:1218-1222)
    PF_OR(pf_norm_q8k(b.X, nb - 1, 1, E, a.out_norm, a.eps, b.qs, b.dd, b.bs, st), "the output norm");
    PF_OR(launch_mv_dev(a.output.p, a.output.type, a.vocab, E, 1, b.qs, b.dd, b.bs, a.logits, 0, 1.f, errw, st), "the output product");
    CUDA_OR(cudaMemcpyAsync(logits, a.logits, static_cast<size_t>(a.vocab) * 4, cudaMemcpyDeviceToHost, st), "logits download");
  }
  CUDA_OR(cudaStreamSynchronize(st), "running the batch");
  int code = 0;
  CUDA_OR(cudaMemcpy(&code, errw, 4, cudaMemcpyDeviceToHost), "reading the device error word");
  if (code) { errf(err, errlen, "device error %d in the batched prompt path", code); cudaMemset(errw, 0, 4096); return 1; }
  if (logits && a.logit_scale != 1.0f)
    for (int i = 0; i < a.vocab; ++i) logits[i] /= a.logit_scale;
  m->pos += nb;
  return 0;
}

int clb200_model_set_batch(clb200_model *m, int tokens) {
  if (!m || tokens < 1 || tokens > PF_MAX_BATCH) return 1;
  m->pf_cap = tokens;
  return 0;
}

int clb200_model_prefill(clb200_model *m, const int *tokens, int n, float *logits, char *err, size_t errlen) {
  if (!m) { errf(err, errlen, "no model"); return 1; }
  const FwdArgs &a = m->args;
  if (n < 1 || !tokens) { errf(err, errlen, "nothing to feed"); return 1; }
  if (m->pos + n > a.ctx) { errf(err, errlen, "the context is full (%d tokens)", a.ctx); return 1; }
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= a.vocab) { errf(err, errlen, "token %d is outside the vocabulary", tokens[i]); return 1; }
  if (m->pos + n > PF_MAX_CTX) { errf(err, errlen, "the batched prompt path takes at most %d positions", PF_MAX_CTX); return 1; }
  cudaSetDevice(m->device);
  const int cap = m->pf_cap;
  if (n > 1 && m->pf_alloc < cap) {
    if (m->pf) { CUDA_OR(cudaStreamSynchronize(m->stream), "waiting for the device"); cudaFree(m->pf); m->pf = nullptr; m->pf_alloc = 0; }
    CUDA_OR(cudaMalloc(&m->pf, pf_layout(a, cap, nullptr).total), "allocating the batched prompt buffers");
    m->pf_alloc = cap;
  }
  for (int i = 0; i < n; i += cap) {   // batches of cap tokens; a batch of one is a step (c/src/forward.c:1263-1266)
    const int nb = std::min(cap, n - i);
    float *lg = i + nb == n ? logits : nullptr;
    if (nb == 1) {
      if (clb200_model_step(m, tokens[i], lg, nullptr, nullptr, nullptr, err, errlen)) return 1;
    } else if (prefill_batch(m, tokens + i, nb, lg, err, errlen)) {
      return 1;
    }
  }
  return 0;
}

}  // extern "C"
