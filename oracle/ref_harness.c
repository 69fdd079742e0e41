/*
 * TEST INFRASTRUCTURE ONLY: a harness around the reference engine compiled from its own sources (oracle/Makefile builds it with
 * them into oracle/_ref/libclref.so). It includes the reference's c/src/forward.c, as the reference's c/test/test_attention.c:4
 * does, to reach its static rmsnorm and dotf, and drives the reference's MoE arithmetic in the order of the forward pass:
 *   one token   c/src/forward.c:949-1033 (rank-order combine),
 *   a batch     c/src/forward.c:1132-1210 (experts in order of first appearance, each over its tokens in ascending order).
 * The glue below (loops, buffers) is this repository's own; every number it produces comes from the reference's functions:
 * rmsnorm, dotf, expf, cl_xq_quantize and cl_matvec_batch (the CPU backend with its thread pool).
 */
#include "forward.c"

typedef struct {
  const float *ffn_norm;
  const float *router;
  uint32_t gate_type, up_type, down_type;
  const uint8_t *gate, *up, *down;
  uint64_t gate_slab, up_slab, down_slab;
  int E, FF, NE, K, norm_topk;
  float resid_scale, rms_eps;
} ref_layer;

void ref_rmsnorm(float *out, const float *x, const float *w, int n, float eps) { rmsnorm(out, x, w, n, eps); }
float ref_dotf(const float *a, const float *b, int n) { return dotf(a, b, n); }

/* softmax, top-k by repeated arg-max (ties to the lower id), renormalisation: the statements of c/src/forward.c:954-984 */
static void route_one(float *rl, int NE, int K, int norm_topk, int *sel, float *wt) {
  float mx = rl[0];
  for (int e = 1; e < NE; e++) if (rl[e] > mx) mx = rl[e];
  double sum = 0;
  for (int e = 0; e < NE; e++) { rl[e] = expf(rl[e] - mx); sum += rl[e]; }
  for (int e = 0; e < NE; e++) rl[e] = (float)(rl[e] / sum);
  char used[4096] = {0};
  for (int k = 0; k < K; k++) {
    int best = -1;
    for (int e = 0; e < NE; e++) if (!used[e] && (best < 0 || rl[e] > rl[best])) best = e;
    used[best] = 1; sel[k] = best; wt[k] = rl[best];
  }
  if (norm_topk) { float z = 0; for (int k = 0; k < K; k++) z += wt[k]; if (z > 0) for (int k = 0; k < K; k++) wt[k] /= z; }
}

void ref_route(float *rl, int NE, int K, int norm_topk, int *sel, float *wt) { route_one(rl, NE, K, norm_topk, sel, wt); }

static int decode_one(const ref_layer *L, float *x, int *sel, float *wt) {
  const int E = L->E, FF = L->FF, K = L->K;
  float *xn = malloc((size_t)E * 4), *rl = malloc((size_t)L->NE * 4), *moe = calloc((size_t)E, 4);
  float *hg = malloc((size_t)K * FF * 4), *hu = malloc((size_t)K * FF * 4), *hd = malloc((size_t)K * E * 4);
  cl_xq xq = {0}, *xqf = calloc((size_t)K, sizeof(cl_xq));
  int ok = xn && rl && moe && hg && hu && hd && xqf && cl_xq_init(&xq, E);
  for (int k = 0; ok && k < K; k++) ok = cl_xq_init(&xqf[k], FF);
  if (ok) {
    rmsnorm(xn, x, L->ffn_norm, E, L->rms_eps);
    for (int e = 0; e < L->NE; e++) rl[e] = dotf(L->router + (size_t)e * E, xn, E);
    route_one(rl, L->NE, K, L->norm_topk, sel, wt);
    cl_xq_quantize(&xq, xn);
    cl_mv j[64];
    for (int k = 0; k < K; k++) {
      j[2 * k] = (cl_mv){L->gate_type, L->gate + (size_t)sel[k] * L->gate_slab, FF, E, xn, &xq, hg + (size_t)k * FF, 1, 0, 0};
      j[2 * k + 1] = (cl_mv){L->up_type, L->up + (size_t)sel[k] * L->up_slab, FF, E, xn, &xq, hu + (size_t)k * FF, 1, 0, 0};
    }
    cl_matvec_batch(j, 2 * K);
    for (int k = 0; k < K; k++) {
      float *g = hg + (size_t)k * FF, *u = hu + (size_t)k * FF;
      for (int i = 0; i < FF; i++) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
      cl_xq_quantize(&xqf[k], g);
      j[k] = (cl_mv){L->down_type, L->down + (size_t)sel[k] * L->down_slab, E, FF, g, &xqf[k], hd + (size_t)k * E, 1, 0, 0};
    }
    cl_matvec_batch(j, K);
    for (int k = 0; k < K; k++) for (int i = 0; i < E; i++) moe[i] += wt[k] * hd[(size_t)k * E + i];
    for (int i = 0; i < E; i++) x[i] += L->resid_scale * moe[i];
  }
  for (int k = 0; xqf && k < K; k++) cl_xq_free(&xqf[k]);
  cl_xq_free(&xq); free(xqf); free(xn); free(rl); free(moe); free(hg); free(hu); free(hd);
  return ok ? 0 : 1;
}

/* The batched block's dispatch, statement for statement: todo[] = the experts in order of first appearance over the
 * (token, rank) slots (c/src/forward.c:1162-1163); for todo[i], who[] / wgt[] = the tokens that chose it, ascending, with the
 * weight of the first slot naming it (:1188-1189). Here the per-expert lists are laid end to end: todo[i]'s entries are
 * [woff[i], woff[i+1]) of who / wgt. Returns the number of experts in todo. */
static int dispatch_lists(const int *sel, const float *wt, int nb, int NU, int NE, int *todo, int *woff, int *who, float *wgt) {
  char *seen = calloc((size_t)NE, 1);
  int n_todo = 0;
  if (!seen) return -1;
  for (int b = 0; b < nb; b++) for (int k = 0; k < NU; k++) { const int e = sel[(size_t)b * NU + k]; if (!seen[e]) { seen[e] = 1; todo[n_todo++] = e; } }
  int ni = 0;
  for (int i = 0; i < n_todo; i++) {
    const int e = todo[i];
    woff[i] = ni;
    for (int b = 0; b < nb; b++) for (int k = 0; k < NU; k++) if (sel[(size_t)b * NU + k] == e) { who[ni] = b; wgt[ni] = wt[(size_t)b * NU + k]; ni++; break; }
  }
  woff[n_todo] = ni;
  free(seen);
  return n_todo;
}

int ref_dispatch(const int *sel, const float *wt, int nb, int NU, int NE, int *todo, int *woff, int *who, float *wgt) {
  return dispatch_lists(sel, wt, nb, NU, NE, todo, woff, who, wgt);
}

/* Routing alone for T tokens (the batched block's route step and per-token softmax/top-k, c/src/forward.c:1065-1072 and
 * :1135-1157): sel / wt [T x K]. */
int ref_route_batch(const ref_layer *L, const float *X, int T, int *sel, float *wt) {
  float *xn = malloc((size_t)L->E * 4), *rl = malloc((size_t)L->NE * 4);
  if (!xn || !rl) { free(xn); free(rl); return 1; }
  for (int b = 0; b < T; b++) {
    rmsnorm(xn, X + (size_t)b * L->E, L->ffn_norm, L->E, L->rms_eps);
    for (int e = 0; e < L->NE; e++) rl[e] = dotf(L->router + (size_t)e * L->E, xn, L->E);
    route_one(rl, L->NE, L->K, L->norm_topk, sel + (size_t)b * L->K, wt + (size_t)b * L->K);
  }
  free(xn); free(rl);
  return 0;
}

static int batch(const ref_layer *L, float *X, int nb, int *sel, float *wt) {
  const int E = L->E, FF = L->FF, NE = L->NE, NU = L->K;
  float *XN = malloc((size_t)nb * E * 4), *XG = malloc((size_t)nb * E * 4), *MOE = calloc((size_t)nb * E, 4), *rl = malloc((size_t)NE * 4);
  float *HG = malloc((size_t)nb * FF * 4), *HU = malloc((size_t)nb * FF * 4), *HDE = malloc((size_t)nb * E * 4);
  cl_xq *xqe = calloc((size_t)nb, sizeof(cl_xq)), *xqf = calloc((size_t)nb, sizeof(cl_xq)), *sub = calloc((size_t)nb, sizeof(cl_xq));
  int *who = malloc((size_t)nb * NU * sizeof(int)), *todo = malloc((size_t)NE * sizeof(int)), *woff = malloc((size_t)(NE + 1) * sizeof(int));
  float *wgt = malloc((size_t)nb * NU * 4);
  int ok = XN && XG && MOE && rl && HG && HU && HDE && xqe && xqf && sub && who && todo && woff && wgt;
  for (int b = 0; ok && b < nb; b++) ok = cl_xq_init(&xqe[b], E) && cl_xq_init(&xqf[b], FF);
  if (ok) {
    for (int b = 0; b < nb; b++) {   /* route_task (c/src/forward.c:1065-1072), then the per-token softmax/top-k (:1135-1157) */
      float *xn = XN + (size_t)b * E;
      rmsnorm(xn, X + (size_t)b * E, L->ffn_norm, E, L->rms_eps);
      cl_xq_quantize(&xqe[b], xn);
      for (int e = 0; e < NE; e++) rl[e] = dotf(L->router + (size_t)e * E, xn, E);
      route_one(rl, NE, NU, L->norm_topk, sel + (size_t)b * NU, wt + (size_t)b * NU);
    }
    const int n_todo = dispatch_lists(sel, wt, nb, NU, NE, todo, woff, who, wgt);
    ok = n_todo >= 0;
    for (int i = 0; i < n_todo; i++) {
      const int e = todo[i], ni = woff[i + 1] - woff[i];
      const int *whoi = who + woff[i];
      const float *wgti = wgt + woff[i];
      for (int t = 0; t < ni; t++) { sub[t] = xqe[whoi[t]]; memcpy(XG + (size_t)t * E, XN + (size_t)whoi[t] * E, (size_t)E * 4); }
      cl_mv j[2] = {{L->gate_type, L->gate + (size_t)e * L->gate_slab, FF, E, XG, sub, HG, ni, (size_t)E, (size_t)FF},
                    {L->up_type, L->up + (size_t)e * L->up_slab, FF, E, XG, sub, HU, ni, (size_t)E, (size_t)FF}};
      cl_matvec_batch(j, 2);
      for (int t = 0; t < ni; t++) {
        float *hg = HG + (size_t)t * FF, *hu = HU + (size_t)t * FF;
        for (int q = 0; q < FF; q++) hg[q] = hg[q] / (1.0f + expf(-hg[q])) * hu[q];
        cl_xq_quantize(&xqf[t], hg);
      }
      cl_mv d = {L->down_type, L->down + (size_t)e * L->down_slab, E, FF, HG, xqf, HDE, ni, (size_t)FF, (size_t)E};
      cl_matvec_batch(&d, 1);
      for (int t = 0; t < ni; t++) { float *m = MOE + (size_t)whoi[t] * E; const float *h = HDE + (size_t)t * E; for (int q = 0; q < E; q++) m[q] += wgti[t] * h[q]; }
    }
    for (size_t i = 0; i < (size_t)nb * E; i++) X[i] += L->resid_scale * MOE[i];
  }
  for (int b = 0; b < nb; b++) { if (xqe) cl_xq_free(&xqe[b]); if (xqf) cl_xq_free(&xqf[b]); }
  free(XN); free(XG); free(MOE); free(rl); free(HG); free(HU); free(HDE); free(xqe); free(xqf); free(sub); free(who); free(todo); free(woff); free(wgt);
  return ok ? 0 : 1;
}

/* T tokens through one MoE layer (x [T x E] in place); sel/wt [T x K]. At most CL_PS_B tokens per batch, like the reference. */
int ref_moe_ffn(const ref_layer *L, float *x, int T, int *sel, float *wt) {
  if (T < 1 || T > CL_PS_B || L->K > 64 || L->NE > 4096) return 1;
  return T == 1 ? decode_one(L, x, sel, wt) : batch(L, x, T, sel, wt);
}

/* ---- the reference's whole forward pass (c/src/forward.h:114-118), for the device step's parity checks ------------------ */
/* Opens a GGUF model with the reference's cl_fwd_open (mapped, no streaming); NULL with err set on failure. */
void *ref_fwd_open(const char *path, int n_ctx, char *err, size_t errlen) {
  cl_fwd *f = calloc(1, sizeof *f);
  if (!f) return NULL;
  if (cl_fwd_open(f, path, n_ctx, NULL, err, errlen)) { free(f); return NULL; }
  return f;
}
/* info[0..7] = n_layer, n_embd, n_vocab, n_expert, n_used, n_ctx_max, pos, head_dim */
void ref_fwd_info(void *h, int *info) {
  const cl_fwd *f = h;
  info[0] = f->n_layer; info[1] = f->n_embd; info[2] = f->n_vocab; info[3] = f->n_expert; info[4] = f->n_used;
  info[5] = f->n_ctx_max; info[6] = f->pos; info[7] = f->head_dim;
}
/* cl_fwd_step: logits [n_vocab]; sel / wt [n_layer * n_used] (may be NULL). */
int ref_fwd_step(void *h, int token, float *logits, int *sel, float *wt, char *err, size_t errlen) {
  cl_fwd *f = h;
  cl_fwd_route rt = {sel, wt, NULL, f->n_layer, f->n_used};
  return cl_fwd_step(f, token, logits, sel && wt ? &rt : NULL, err, errlen);
}
/* cl_fwd_prefill (c/src/forward.h:121): n tokens in batches (run_std); logits [n_vocab] after the last one (may be NULL). */
int ref_fwd_prefill(void *h, const int *tokens, int n, float *logits, char *err, size_t errlen) {
  return cl_fwd_prefill(h, tokens, n, logits, err, errlen);
}
void ref_fwd_close(void *h) {
  if (!h) return;
  cl_fwd_close(h);
  free(h);
}
