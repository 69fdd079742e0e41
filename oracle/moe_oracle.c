/*
 * TEST INFRASTRUCTURE ONLY: the oracle. A plain-C, single-threaded restatement of the Clutor engine's
 * mixture-of-experts feed-forward block, used by tests/, the smoke check and the CPU-baseline leg of
 * bench.py as the checker of the CUDA path. Nothing in the product links or calls this file.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the reference's own
 * known-answer tests (c/test/test_engine.c) and against the reference compiled from its sources
 * (oracle/_ref, built by oracle/Makefile), and tests/golden/ holds fixtures made by the latter.
 *
 * Build flags matter: -std=c11 (no FMA contraction, like the reference's -O2 -std=c11 -mavx2 -mf16c
 * build, c/Makefile:3-9), so every float operation rounds exactly where the reference's does.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ggml tensor type ids (c/src/quant.h:7). */
enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

/* Q8_K activation block: the reference's cl_q8k (c/src/quant.h:22): scale, 256 int8, 16 group sums; 292 bytes. */
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } orc_q8k;

/* Half to single precision from the IEEE 754 binary16 definition (c/src/kernel.c:25-39 is the reference's version). */
float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const int ex = (h >> 10) & 31;
  const uint32_t mant = h & 1023u;
  uint32_t bits;
  if (ex == 31) bits = sign | 0x7f800000u | (mant << 13);
  else if (ex > 0) bits = sign | ((uint32_t)(ex - 15 + 127) << 23) | (mant << 13);
  else if (mant == 0) bits = sign;
  else {                                   /* subnormal: value = mant * 2^-24, renormalised */
    int shift = 0;
    uint32_t m = mant;
    while (!(m & 1024u)) { m <<= 1; shift++; }
    bits = sign | ((uint32_t)(127 - 14 - shift) << 23) | ((m & 1023u) << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

uint32_t orc_block_elems(uint32_t type) { return type == T_Q8_0 ? 32 : (type == T_Q4_K || type == T_Q6_K) ? 256 : type == T_F16 || type == T_F32 ? 1 : 0; }
uint32_t orc_block_bytes(uint32_t type) { return type == T_Q8_0 ? 34 : type == T_Q4_K ? 144 : type == T_Q6_K ? 210 : type == T_F16 ? 2 : type == T_F32 ? 4 : 0; }
uint64_t orc_row_bytes(uint32_t type, uint64_t n) { return n / orc_block_elems(type) * orc_block_bytes(type); }

/* The 6-bit (scale, min) of sub-block j of a Q4_K block from its 12 packed bytes: sub-blocks 0-3 keep the low 6 bits of bytes j and
 * j+4; sub-blocks 4-7 take a nibble of byte j+4 plus the top two bits of bytes j-4 / j (ggml's layout; c/src/quant.c:36-40). */
static void q4k_scale_min(const uint8_t *s12, int j, int *sc, int *mn) {
  if (j < 4) { *sc = s12[j] & 63; *mn = s12[j + 4] & 63; }
  else { *sc = (s12[j + 4] & 15) | ((s12[j - 4] >> 6) << 4); *mn = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4); }
}

/* Q4_K block (144 B: d, dmin fp16, 12 scale bytes, 128 nibble bytes): element 64g+l is the low nibble of qs[32g+l], element
 * 64g+32+l its high nibble, in sub-blocks 2g and 2g+1 (c/src/quant.c:54-68). value = d*sc*q - dmin*mn. */
static void deq_q4k(const uint8_t *b, float *y) {
  const float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
  const uint8_t *s12 = b + 4, *qs = b + 16;
  for (int g = 0; g < 4; g++) {
    int sc0, mn0, sc1, mn1;
    q4k_scale_min(s12, 2 * g, &sc0, &mn0);
    q4k_scale_min(s12, 2 * g + 1, &sc1, &mn1);
    const float d0 = d * (float)sc0, m0 = dmin * (float)mn0, d1 = d * (float)sc1, m1 = dmin * (float)mn1;
    for (int l = 0; l < 32; l++) y[64 * g + l] = d0 * (float)(qs[32 * g + l] & 15) - m0;
    for (int l = 0; l < 32; l++) y[64 * g + 32 + l] = d1 * (float)(qs[32 * g + l] >> 4) - m1;
  }
}

/* Unpacks a Q6_K block (210 B: ql[128], qh[64], int8 scales[16], fp16 d) to its 256 signed 6-bit values (-32..31): in each half of
 * 128, element 32c+l takes a nibble of ql (low for c=0,1; high for c=2,3; byte l or l+32) and two bits (2c..2c+1) of qh[l]
 * (c/src/quant.c:87-105). Group g of 16 values uses scales[g]. */
static void unpack_q6k(const uint8_t *b, int8_t *q) {
  const uint8_t *ql = b, *qh = b + 128;
  for (int h = 0; h < 2; h++) {
    for (int l = 0; l < 32; l++) {
      const int lo0 = ql[64 * h + l], lo1 = ql[64 * h + 32 + l], hi = qh[32 * h + l];
      q[128 * h + l] = (int8_t)(((lo0 & 15) | ((hi & 3) << 4)) - 32);
      q[128 * h + 32 + l] = (int8_t)(((lo1 & 15) | (((hi >> 2) & 3) << 4)) - 32);
      q[128 * h + 64 + l] = (int8_t)(((lo0 >> 4) | (((hi >> 4) & 3) << 4)) - 32);
      q[128 * h + 96 + l] = (int8_t)(((lo1 >> 4) | (((hi >> 6) & 3) << 4)) - 32);
    }
  }
}
static void deq_q6k(const uint8_t *b, float *y) {
  int8_t q[256];
  unpack_q6k(b, q);
  const int8_t *sc = (const int8_t *)(b + 192);
  const float d = orc_f16_to_f32(rd16(b + 208));
  for (int i = 0; i < 256; i++) y[i] = d * (float)sc[i / 16] * (float)q[i];
}

/* Dequantizes n elements of one row. */
void orc_dequant_row(uint32_t type, const void *src, float *dst, int n) {
  const uint8_t *p = src;
  if (type == T_F32) { memcpy(dst, src, (size_t)n * 4); return; }
  if (type == T_F16) { for (int i = 0; i < n; i++) dst[i] = orc_f16_to_f32(rd16(p + 2 * i)); return; }
  if (type == T_Q8_0) {
    for (int b = 0; b < n / 32; b++) {
      const float d = orc_f16_to_f32(rd16(p + 34 * b));
      for (int j = 0; j < 32; j++) dst[32 * b + j] = (float)(int8_t)p[34 * b + 2 + j] * d;
    }
    return;
  }
  if (type == T_Q4_K) { for (int b = 0; b < n / 256; b++) deq_q4k(p + 144 * b, dst + 256 * b); return; }
  if (type == T_Q6_K) { for (int b = 0; b < n / 256; b++) deq_q6k(p + 210 * b, dst + 256 * b); return; }
  memset(dst, 0, (size_t)n * 4);
}

/* Q8_K quantization of n floats (n a multiple of 256): per block d = amax/127, q = round-half-away(x/d computed as x*(1/d)),
 * bsums = sums of 16 (c/src/quant.c:195-206). */
void orc_q8k_quantize(const float *x, int n, orc_q8k *out) {
  for (int b = 0; b < n / 256; b++) {
    const float *v = x + 256 * b;
    float amax = 0;
    for (int j = 0; j < 256; j++) { const float a = fabsf(v[j]); if (a > amax) amax = a; }
    const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
    out[b].d = d;
    for (int j = 0; j < 256; j++) out[b].qs[j] = (int8_t)roundf(v[j] * id);
    for (int g = 0; g < 16; g++) { int s = 0; for (int j = 0; j < 16; j++) s += out[b].qs[16 * g + j]; out[b].bsums[g] = (int16_t)s; }
  }
}

/* One weight row times one activation. K-quants: exact integer sums per 256-block on Q8_K activations, then
 * sum += yd*(d*sumi - dmin*summs) (Q4_K) or sum += (d*yd)*sumi (Q6_K), blocks in order (c/src/quant.c:255-287, 329-360, 832-846).
 * Q8_0 and float types: the reference's float path, a block-local float sum added to the row total (c/src/quant.c:889-902). */
float orc_dot_row(uint32_t type, const void *row, int cols, const orc_q8k *xq, const float *xf) {
  const uint8_t *p = row;
  if (type == T_Q4_K) {
    float sum = 0;
    for (int i = 0; i < cols / 256; i++) {
      const uint8_t *b = p + 144 * i, *qs = b + 16;
      const orc_q8k *y = &xq[i];
      int32_t sumi = 0, summs = 0;
      for (int g = 0; g < 4; g++) {
        int sc0, mn0, sc1, mn1;
        q4k_scale_min(b + 4, 2 * g, &sc0, &mn0);
        q4k_scale_min(b + 4, 2 * g + 1, &sc1, &mn1);
        int32_t a = 0, c = 0;
        for (int l = 0; l < 32; l++) { a += (qs[32 * g + l] & 15) * y->qs[64 * g + l]; c += (qs[32 * g + l] >> 4) * y->qs[64 * g + 32 + l]; }
        sumi += sc0 * a + sc1 * c;
        summs += mn0 * (y->bsums[4 * g] + y->bsums[4 * g + 1]) + mn1 * (y->bsums[4 * g + 2] + y->bsums[4 * g + 3]);
      }
      sum += y->d * (orc_f16_to_f32(rd16(b)) * (float)sumi - orc_f16_to_f32(rd16(b + 2)) * (float)summs);
    }
    return sum;
  }
  if (type == T_Q6_K) {
    float sum = 0;
    for (int i = 0; i < cols / 256; i++) {
      const uint8_t *b = p + 210 * i;
      int8_t q[256];
      unpack_q6k(b, q);
      const int8_t *sc = (const int8_t *)(b + 192);
      int32_t sumi = 0;
      for (int g = 0; g < 16; g++) { int32_t t = 0; for (int l = 0; l < 16; l++) t += q[16 * g + l] * xq[i].qs[16 * g + l]; sumi += sc[g] * t; }
      sum += orc_f16_to_f32(rd16(b + 208)) * xq[i].d * (float)sumi;
    }
    return sum;
  }
  const uint32_t bl = orc_block_elems(type), bb = orc_block_bytes(type);
  if (!bl) return 0;
  if (type == T_F32) { const float *w = row; float s = 0; for (int i = 0; i < cols; i++) s += w[i] * xf[i]; return s; }
  float acc = 0, buf[256];
  for (int c = 0; c < cols; c += (int)bl) {
    orc_dequant_row(type, p + (size_t)(c / (int)bl) * bb, buf, (int)bl);
    float s = 0;
    for (uint32_t i = 0; i < bl; i++) s += buf[i] * xf[c + i];
    acc += s;
  }
  return acc;
}

/* RMSNorm with a double-precision sum of squares, scaled as (x*s)*w (c/src/forward.c:412-417). */
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
  double ss = 0;
  for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
  const float s = 1.0f / sqrtf((float)(ss / (double)n) + eps);
  for (int i = 0; i < n; i++) out[i] = x[i] * s * w[i];
}

/* The router's dot product: eight strided float partial sums, combined ((0+1)+(2+3))+((4+5)+(6+7)), then a scalar tail
 * (c/src/forward.c:574-581). */
float orc_dotf(const float *a, const float *b, int n) {
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= n; i += 8) for (int l = 0; l < 8; l++) s[l] += a[i + l] * b[i + l];
  float t = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
  for (; i < n; i++) t += a[i] * b[i];
  return t;
}

/* Softmax over NE logits (float exp of logit-max, double sum, double divide), the K best by repeated arg-max with ties to the lower
 * id, optionally renormalised by their float sum (c/src/forward.c:954-984). logits is overwritten with the probabilities. */
void orc_route(float *rl, int NE, int K, int norm_topk, int *sel, float *wt) {
  float mx = rl[0];
  for (int e = 1; e < NE; e++) if (rl[e] > mx) mx = rl[e];
  double sum = 0;
  for (int e = 0; e < NE; e++) { rl[e] = expf(rl[e] - mx); sum += rl[e]; }
  for (int e = 0; e < NE; e++) rl[e] = (float)(rl[e] / sum);
  char *used = calloc((size_t)NE, 1);
  for (int k = 0; k < K; k++) {
    int best = -1;
    for (int e = 0; e < NE; e++) if (!used[e] && (best < 0 || rl[e] > rl[best])) best = e;
    used[best] = 1; sel[k] = best; wt[k] = rl[best];
  }
  free(used);
  if (norm_topk) { float z = 0; for (int k = 0; k < K; k++) z += wt[k]; if (z > 0) for (int k = 0; k < K; k++) wt[k] /= z; }
}

/* SMART-ROUTE (c/src/route.c:13-52): the experts ranked by their double softmax probability (exp of logit minus the
 * maximum, divided by the sum taken in expert order), best first and ties to the lower id; the first K are the plain choice.
 * With smart_on and a residency array, the ranks below J and the resident experts stay; each other rank, in rank order,
 * takes the lowest rank j < M (clamped to [K, E]) whose expert is resident, unused and no more than tau below it in
 * probability, else keeps its own expert. Returns -1 for E or K out of range (E > 1024, K > 32, K > E, or < 1), else 0. */
typedef struct { int id; double p; } orc_ranked;
static int orc_rank_cmp(const void *a, const void *b) {
  const orc_ranked *x = (const orc_ranked *)a, *y = (const orc_ranked *)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  return (x->id > y->id) - (x->id < y->id);
}
int orc_smart_route(const float *logits, int E, int K, int smart_on, int J, int M, double tau, const uint8_t *resident,
                    int *selected, int *substituted, double *dropped, double *max_delta) {
  if (E < 1 || E > 1024 || K < 1 || K > 32 || K > E) return -1;
  orc_ranked rk[1024];
  double mx = logits[0], sum = 0.0;
  for (int i = 1; i < E; i++) mx = logits[i] > mx ? logits[i] : mx;
  for (int i = 0; i < E; i++) { rk[i].id = i; rk[i].p = exp((double)logits[i] - mx); sum += rk[i].p; }
  for (int i = 0; i < E; i++) rk[i].p = rk[i].p / sum;
  qsort(rk, (size_t)E, sizeof rk[0], orc_rank_cmp);
  *substituted = 0; *dropped = 0.0; *max_delta = 0.0;
  for (int k = 0; k < K; k++) selected[k] = rk[k].id;
  if (!smart_on || !resident) return 0;
  if (J < 0) J = 0;
  if (J > K) J = K;
  if (M < K) M = K;
  if (M > E) M = E;
  unsigned char used[1024];
  memset(used, 0, sizeof used);
  int cold[32], nc = 0;
  for (int k = 0; k < K; k++) {
    if (k < J || resident[rk[k].id]) used[rk[k].id] = 1;
    else cold[nc++] = k;
  }
  for (int c = 0; c < nc; c++) {
    const int k = cold[c];
    int j = 0;
    for (; j < M; j++)
      if (j != k && !used[rk[j].id] && resident[rk[j].id] && !(rk[k].p - rk[j].p > tau)) break;
    if (j == M) { used[rk[k].id] = 1; continue; }
    const double d = rk[k].p - rk[j].p;
    used[rk[j].id] = 1;
    selected[k] = rk[j].id;
    *substituted += 1;
    *dropped += d;
    if (d > *max_delta) *max_delta = d;
  }
  return 0;
}

static float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

/* One MoE layer, mirroring the reference's types: fused expert tensors with rows-per-expert and byte slabs (c/src/forward.h:18-29). */
typedef struct {
  const float *ffn_norm;        /* [E] */
  const float *router;          /* [NE x E] */
  uint32_t gate_type, up_type, down_type;
  const uint8_t *gate, *up, *down;
  uint64_t gate_slab, up_slab, down_slab;   /* bytes of one expert */
  int E, FF, NE, K, norm_topk;
  float resid_scale, rms_eps;
} orc_layer;

static int is_kquant(uint32_t t) { return t == T_Q4_K || t == T_Q6_K; }

/* T tokens through the layer, x [T x E] updated in place. sel/wt [T x K] receive the routing. T == 1 follows the one-token block
 * (c/src/forward.c:949-1033: experts combined in rank order); T > 1 the batched block (c/src/forward.c:1132-1210: experts in
 * order of first appearance, each over its tokens in ascending order). Returns 0, or 1 when memory runs out. */
int orc_moe_ffn(const orc_layer *L, float *x, int T, int *sel, float *wt) {
  const int E = L->E, FF = L->FF, NE = L->NE, K = L->K;
  float *xn = malloc((size_t)T * E * 4), *rl = malloc((size_t)NE * 4), *moe = calloc((size_t)T * E, 4);
  float *hg = malloc((size_t)FF * 4), *hu = malloc((size_t)FF * 4), *hd = malloc((size_t)E * 4);
  orc_q8k *xq = malloc((size_t)T * (E / 256) * sizeof(orc_q8k)), *hq = malloc((size_t)(FF / 256) * sizeof(orc_q8k));
  int *order = malloc((size_t)NE * sizeof(int)); char *seen = calloc((size_t)NE, 1);
  if (!xn || !rl || !moe || !hg || !hu || !hd || !xq || !hq || !order || !seen) { free(xn); free(rl); free(moe); free(hg); free(hu); free(hd); free(xq); free(hq); free(order); free(seen); return 1; }
  for (int t = 0; t < T; t++) {
    float *xt = xn + (size_t)t * E;
    orc_rmsnorm(xt, x + (size_t)t * E, L->ffn_norm, E, L->rms_eps);
    for (int e = 0; e < NE; e++) rl[e] = orc_dotf(L->router + (size_t)e * E, xt, E);
    orc_route(rl, NE, K, L->norm_topk, sel + (size_t)t * K, wt + (size_t)t * K);
    orc_q8k_quantize(xt, E, xq + (size_t)t * (E / 256));
  }
  /* expert order: rank order for one token, first appearance for a batch */
  int n_order = 0;
  for (int t = 0; t < T; t++) for (int k = 0; k < K; k++) { const int e = sel[(size_t)t * K + k]; if (!seen[e]) { seen[e] = 1; order[n_order++] = e; } }
  for (int i = 0; i < n_order; i++) {
    const int e = order[i];
    const uint8_t *g = L->gate + (size_t)e * L->gate_slab, *u = L->up + (size_t)e * L->up_slab, *dn = L->down + (size_t)e * L->down_slab;
    const uint64_t grb = orc_row_bytes(L->gate_type, (uint64_t)E), urb = orc_row_bytes(L->up_type, (uint64_t)E), drb = orc_row_bytes(L->down_type, (uint64_t)FF);
    for (int t = 0; t < T; t++) {
      int slot = -1;
      for (int k = 0; k < K; k++) if (sel[(size_t)t * K + k] == e) { slot = k; break; }
      if (slot < 0) continue;
      const float *xt = xn + (size_t)t * E;
      const orc_q8k *xqt = xq + (size_t)t * (E / 256);
      for (int r = 0; r < FF; r++) {
        hg[r] = orc_dot_row(L->gate_type, g + (size_t)r * grb, E, xqt, xt);
        hu[r] = orc_dot_row(L->up_type, u + (size_t)r * urb, E, xqt, xt);
      }
      for (int r = 0; r < FF; r++) hg[r] = silu_mul(hg[r], hu[r]);
      if (is_kquant(L->down_type)) orc_q8k_quantize(hg, FF, hq);
      for (int r = 0; r < E; r++) hd[r] = orc_dot_row(L->down_type, dn + (size_t)r * drb, FF, hq, hg);
      const float w = wt[(size_t)t * K + slot];
      float *m = moe + (size_t)t * E;
      for (int r = 0; r < E; r++) m[r] += w * hd[r];
    }
  }
  for (size_t i = 0; i < (size_t)T * E; i++) x[i] += L->resid_scale * moe[i];
  free(xn); free(rl); free(moe); free(hg); free(hu); free(hd); free(xq); free(hq); free(order); free(seen);
  return 0;
}
