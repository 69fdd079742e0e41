// The whole-model one-token step as ONE persistent kernel: the reference's cl_fwd_step (c/src/forward.c:878-1040) for the
// mixture-of-experts transformers (olmoe, qwen3moe, granitemoe) on one B200.
//
// One CTA per SM (G CTAs, a cooperative launch, so all are resident), 512 threads. Work that crosses CTAs goes through
// global memory behind one grid barrier counter (bounded waits; any CTA's error ends every CTA's wait). Per layer:
//   A  attention input: x (global) -> rmsnorm -> Q8_K blocks (every CTA); this CTA's rows of the stacked [wq; wk; wv]
//      from shared memory (exact integer block sums, the reference's float block terms in block order)       | barrier
//   B  attention, one CTA per query head and no exchange between CTAs: QK-norm and rotary embedding of its query and of
//      its key/value head's new key (c/src/forward.c:905-915), the new key and value into the half-precision cache
//      (kv_put, :563-572, by the group's first head), the reference's dotf_h against every position, then the softmax
//      and weighted values in the reference's order: per 256-position chunk, merged, when a group has 2..16 query heads
//      and the context is 64 positions or more (c/src/forward.c:665-737), else over every position (:584-627) | barrier
//   C  attention output: Q8_K of the attention vector (every CTA); this CTA's rows of wo; x += resid * wo att | barrier
//   D  mixture of experts as the one-token MoE kernel (decode.cu) does it: rmsnorm, router (the reference's dotf), the
//      experts ranked by logit and this CTA's share of the first K sent out at once (bulk copies of gate/up and down rows
//      into shared memory), then softmax, the probability order (a slot fetches again where a tie moves an expert out of
//      the top k), renormalisation, the gate/up rows, SwiGLU                                                  | barrier
//      the Q8_K blocks of every expert's hg, this CTA's down rows, x += resid * sum_k wt_k hd_k in rank order  | barrier
// then the output norm and this CTA's rows of the output matrix, streamed through shared memory, their logits and the
// greedy arg-max (lowest id on ties, c/src/main.c:349-350). The last CTA out advances the sequence state.
//
// Weights never wait on activations: a layer's dense rows (wq, wk, wv, wo) are copied into shared memory while the
// previous layer's down rows compute, and its router rows as soon as the previous layer's router products are formed.
// The code a layer runs is kept small (the block dot products, quantizers and transcendental steps are out-of-line
// functions): a layer executes every phase once, so code that outgrows the SM's instruction caches is fetched again
// for every layer.
#include "common.cuh"
#include "fwd.cuh"
#include "modelops.cuh"
#include "rowdot.cuh"

namespace clb {
namespace {

constexpr int NW = FWD_THREADS / 32;
constexpr int RW = NW - 1;   // the router warp

CLB_DEV int ld_volatile(const int *p) { return *reinterpret_cast<const volatile int *>(p); }

// ---- steps used in several phases ---------------------------------------------------------------------------------------
// The block dot of the per-layer phases is one out-of-line function: one copy of its code instead of five inlined ones
// (the kernel's code does not stay in the instruction caches from one layer to the next; measured 467.6 against 466.4
// tokens/s). The output matrix's hot loop keeps an inlined, unrolled copy.
__device__ __noinline__ float blk_dot(uint32_t type, const uint8_t *row, int blk, const int8_t *qs, const int16_t *bs,
                                      const float *dd, int ablk) {
  return kq_block_s(type, row, blk, SmemAct{qs, bs, dd}, ablk);
}
CLB_DEV float blk_dot_fast(uint32_t type, const uint8_t *row, int blk, const int8_t *qs, const int16_t *bs,
                                           const float *dd, int ablk) {
  return kq_block_s<false>(type, row, blk, SmemAct{qs, bs, dd}, ablk);
}
CLB_DEV void quant_smem(const float *x, int n, int8_t *qs, float *dd, int16_t *bs, int warp, int nwarps, int lane) {
  q8k_quantize_block(x, n, qs, dd, bs, warp, nwarps, lane, true);
}
CLB_DEV void quant_global(const float *src, int nblocks, int8_t *qs, float *dd, int16_t *bs, int warp, int nwarps,
                                          int lane) {
  q8k_quantize_global<2>(src, nblocks, qs, dd, bs, warp, nwarps, lane, true);
}
CLB_DEV float exp_cr(float x) { return expf_cr(x); }
CLB_DEV float swiglu(float g, float u) { return silu_mul(g, u); }

// The block of one grid barrier: every CTA arrives, then waits for all G (bounded; returns early when any CTA has
// recorded an error). Returns false on a timeout or a recorded error.
struct Grid {
  uint32_t *ctr;
  int *err;
  int *s_ok;      // shared: the barrier's verdict for the whole CTA
  uint32_t G, gen;
  CLB_DEV bool sync() {
    __syncthreads();
    if (threadIdx.x == 0) {
      ++gen;
      red_release_add(ctr, 1u);
      const uint32_t target = gen * G;
      bool ok = false;
#pragma unroll 1
      for (uint32_t i = 0; i < SPIN_LIMIT; ++i) {
        if (ld_acquire(ctr) >= target) { ok = true; break; }
        if ((i & 127) == 127 && ld_volatile(err)) break;
        if (i > 4096) __nanosleep(64);
      }
      if (!ok) set_error(err, ERR_WAIT_GRID);
      *s_ok = ok && !ld_volatile(err);
    }
    __syncthreads();
    return *s_ok != 0;
  }
};

// rmsnorm (c/src/forward.c:412-417) of the n floats at x (global, written by other CTAs) with weights w: xn (shared) =
// x * (1 / sqrtf(mean(x^2) + eps)) * w, the mean of squares in double. red: NW doubles of shared scratch.
CLB_DEV void rmsnorm_to_smem(const float *x, const float *w, float *xn, int n, float eps, double *red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int XV = (4096 / 4 + FWD_THREADS - 1) / FWD_THREADS;
  float4 xv[XV];
  double ss = 0.0;
#pragma unroll
  for (int u = 0; u < XV; ++u) {
    const int i = (tid + u * FWD_THREADS) * 4;
    if (i < n) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + i));
      xv[u] = v;
      ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  double tot = 0.0;
#pragma unroll
  for (int k = 0; k < NW; ++k) tot += red[k];
  const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / static_cast<double>(n)), eps)));
#pragma unroll
  for (int u = 0; u < XV; ++u) {
    const int i = (tid + u * FWD_THREADS) * 4;
    if (i < n) {
      const float4 v = xv[u], g = __ldg(reinterpret_cast<const float4 *>(w + i));
      reinterpret_cast<float4 *>(xn + i)[0] = make_float4(__fmul_rn(__fmul_rn(v.x, s), g.x), __fmul_rn(__fmul_rn(v.y, s), g.y),
                                                          __fmul_rn(__fmul_rn(v.z, s), g.z), __fmul_rn(__fmul_rn(v.w, s), g.w));
    }
  }
  __syncthreads();
}

CLB_DEV int lanes_for(int nb) { return nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : nb <= 8 ? 8 : 16; }

// n rows of a K-quant matrix (row i at rows + i * rb, nb 256-blocks each; shared or global memory) times the Q8_K
// vector in shared memory: a group of lanes per row, one lane per block, the block terms added in block order at the
// group's first lane. mode 0: dst[i] = value; mode 1: dst[i] = dst[i] + scale * value (the residual update). Call from
// all threads.
CLB_DEV void gemv_rows(uint32_t type, const uint8_t *rows, uint32_t rb, int nb, int n, const int8_t *qs,
                                       const float *dd, const int16_t *bs, float *dst, int mode, float scale) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int GL = lanes_for(nb), lg = lane & (GL - 1), gpw = 32 / GL, ngroups = NW * gpw, gid = warp * gpw + lane / GL;
  const int base = lane - lg;
  const bool has = lg < nb;
  for (int b0 = 0; b0 < n; b0 += ngroups) {   // the same trip count in every warp
    const int r = b0 + gid;
    const bool valid = r < n;
    float t = 0.f;
    if (valid && has) t = blk_dot(type, rows + static_cast<size_t>(r) * rb, lg, qs, bs, dd, lg);
    float s = 0.f;
    for (int b = 0; b < nb; ++b) s = __fadd_rn(s, __shfl_sync(FULL, t, base + b));
    if (valid && lg == 0) {
      if (mode == 0) __stcg(dst + r, s);
      else dst[r] = __fadd_rn(__ldcg(dst + r), __fmul_rn(scale, s));
    }
  }
}

// The arg-max key of a logit: larger value first, then the lower id.
CLB_DEV unsigned long long argmax_key(float v, int id) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | (0xffffffffu - static_cast<uint32_t>(id));
}

CLB_DEV uint32_t lo16(const void *p) { return static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 15u); }

// Where this CTA's rows [r0[q], r1[q]) of a layer's wq, wk, wv, wo sit in the slots: one segment after another, each
// 32 bytes longer than its rows (the copy starts at the 16-byte boundary at or below the first row).
CLB_DEV uint32_t dense_offset(const FwdLayer &Ly, const int (&r0)[4], const int (&r1)[4], int q) {
  const FwdMat mats[4] = {Ly.wq, Ly.wk, Ly.wv, Ly.wo};
  uint32_t off = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i)
    if (i < q) off += (static_cast<uint32_t>(r1[i] - r0[i]) * mats[i].rb + 32u + 15u) & ~15u;
  return off;
}

// This CTA's rows of a layer's wq, wk, wv, wo, one bulk copy each into its segment of the slots. One thread.
CLB_DEV void issue_dense(const FwdLayer &Ly, uint8_t *slots, uint64_t *bar, const int (&r0)[4], const int (&r1)[4]) {
  const FwdMat mats[4] = {Ly.wq, Ly.wk, Ly.wv, Ly.wo};
  uint32_t total = 0, n16[4];
  const uint8_t *src[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int cnt = r1[q] - r0[q];
    src[q] = mats[q].p + static_cast<size_t>(r0[q]) * mats[q].rb;
    n16[q] = cnt > 0 ? (lo16(src[q]) + static_cast<uint32_t>(cnt) * mats[q].rb + 15u) & ~15u : 0u;
    total += n16[q];
  }
  fence_proxy_async();
  mbar_arrive_expect_tx(bar, total);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    if (n16[q]) bulk_copy_g2s_hint(slots + dense_offset(Ly, r0, r1, q), src[q] - lo16(src[q]), n16[q], bar, l2_evict_first());
}

template <int EPL>
__global__ void __launch_bounds__(FWD_THREADS, 1) fwd_kernel(const FwdArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int E = a.E, FF = a.FF, NE = a.NE, K = a.K;
  constexpr int hd = 32 * EPL;
  const int nb = E / 256, nbd = FF / 256;
  FwdState *st = a.st;

  // [0, K) experts, [K] router rows, [K+1] dense rows, [K+2, K+2+HEAD_STAGES) output stages, [K+2+HEAD_STAGES] the
  // attention head's prefetch
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bars);
  uint64_t *rbar = bars + K, *dbar = bars + K + 1, *hb = bars + K + 2, *abar = bars + K + 2 + HEAD_STAGES;
  float *xn = reinterpret_cast<float *>(smem + a.off_xn);             // [E]
  int8_t *xq_qs = reinterpret_cast<int8_t *>(smem + a.off_xq);        // Q8_K of the current vector (up to n_q wide)
  const int XQW = a.n_q > E ? a.n_q : E;
  int16_t *xq_bs = reinterpret_cast<int16_t *>(smem + a.off_xq + XQW);
  float *xq_d = reinterpret_cast<float *>(smem + a.off_xq + XQW + 2 * (XQW / 16));
  double *s_red = reinterpret_cast<double *>(smem + a.off_misc);      // [NW]
  // [0] barrier verdict, [1] a router copy in flight, [2] the router logits arrived, [3] its parity, [4] the layer of the
  // last attention prefetch (-1: none), [5] a dense copy in flight, [6] its parity, [7] the probability order differs
  // from the logit order
  int *s_flag = reinterpret_cast<int *>(s_red + NW);
  int *s_sel = s_flag + 8;                                             // [32]
  float *s_wt = reinterpret_cast<float *>(s_sel + 32);                 // [32]
  float *s_wn = s_wt + 32;                                             // [32]
  float *probs = s_wn + 32;                                            // [FWD_MAX_NE]
  unsigned long long *s_best = reinterpret_cast<unsigned long long *>(probs + FWD_MAX_NE);   // [NW]
  float *s_lg = reinterpret_cast<float *>(s_best + NW);                // [FWD_MAX_NE] logits, -inf past NE
  int *s_spec = reinterpret_cast<int *>(s_lg + FWD_MAX_NE);           // [32] slot k: the expert it streams
  int *s_slot = s_spec + 32;                                           // [32] rank -> the slot streaming that expert
  int *s_cnt = s_slot + 32;                                            // [32] phases begun on the slot's mbarrier
  int *s_fix = s_cnt + 32;                                             // [32] expert + 1 to fetch into the slot again, or 0
  float *rrows = reinterpret_cast<float *>(smem + a.off_router);      // [nre][E]
  float *rprod = reinterpret_cast<float *>(smem + a.off_rprod);       // [nre][8][E/8 + 4]
  float *terms = reinterpret_cast<float *>(smem + a.off_terms);
  int8_t *hq_qs = reinterpret_cast<int8_t *>(smem + a.off_hq);
  int16_t *hq_bs = reinterpret_cast<int16_t *>(smem + a.off_hq + K * FF);
  float *hq_d = reinterpret_cast<float *>(smem + a.off_hq + K * FF + 2 * (K * FF / 16));
  float *xr = reinterpret_cast<float *>(smem + a.off_xr);
  uint8_t *slots = smem + a.off_slots;     // dense rows of the layer, then the chosen experts' gate/up rows; output stages
  uint8_t *dslots = smem + a.off_dslots;   // down rows of the chosen experts; the attention scratch
  const int GRP = a.n_head / a.n_kv;

  const uint32_t uG = static_cast<uint32_t>(G), uc = static_cast<uint32_t>(c);
  const int j0 = static_cast<int>(FF * uc / uG), j1 = static_cast<int>(FF * (uc + 1) / uG);
  const int i0 = static_cast<int>(E * uc / uG), i1 = static_cast<int>(E * (uc + 1) / uG);
  const int ngu = j1 - j0, nd = i1 - i0;
  const int nre = c < NE ? (NE - c + G - 1) / G : 0;
  const int RS = E / 8 + 4;
  const int nq = a.n_q, nk = a.n_kvw, QKVR = nq + 2 * nk;
  const int qr0 = static_cast<int>(static_cast<uint32_t>(QKVR) * uc / uG), qr1 = static_cast<int>(static_cast<uint32_t>(QKVR) * (uc + 1) / uG);
  // this CTA's rows of wq, wk, wv, wo
  const int dr0[4] = {min(max(qr0, 0), nq), min(max(qr0 - nq, 0), nk), min(max(qr0 - nq - nk, 0), nk), i0};
  const int dr1[4] = {max(min(qr1, nq), dr0[0]), max(min(qr1 - nq, nk), dr0[1]), max(min(qr1 - nq - nk, nk), dr0[2]), i1};

  Grid grid{&st->sync[0], &st->err, &s_flag[0], uG, 0};
  const int pos = st->pos, token = st->token;
  trace_time(a.trace, 30);

  if (tid == 0) {
    for (int s = 0; s < K + 3 + HEAD_STAGES; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    if (nre > 0) {   // layer 0's router rows
      mbar_arrive_expect_tx(rbar, static_cast<uint32_t>(nre) * E * 4u);
      for (int m = 0; m < nre; ++m)
        bulk_copy_g2s_hint(rrows + static_cast<size_t>(m) * E, a.layers[0].router + static_cast<size_t>(c + m * G) * E, E * 4u, rbar, l2_evict_first());
    }
    issue_dense(a.layers[0], slots, dbar, dr0, dr1);   // layer 0's dense rows
    s_flag[1] = nre > 0;
    s_flag[3] = 0;
    for (int k = 0; k < 32; ++k) s_cnt[k] = 0;
    s_flag[4] = -1;
    s_flag[5] = 1;
    s_flag[6] = 0;
  }
  // the token's embedding: this CTA's rows of x
  bool ok = true;
  if (token < 0 || token >= a.vocab || pos < 0 || pos >= a.ctx) {
    if (tid == 0) set_error(&st->err, ERR_BAD_EXPERT);
    ok = false;
  }
  if (ok) {
    embed_row(a.tok_embd, token, E, xn);
    __syncthreads();
    for (int i = i0 + tid; i < i1; i += FWD_THREADS) a.x[i] = a.embed_scale != 1.0f ? __fmul_rn(xn[i], a.embed_scale) : xn[i];
  }
  ok = grid.sync() && ok;
  const int nchunk = (pos + 1 + FWD_ATT_CHUNK - 1) / FWD_ATT_CHUNK;
  const bool grouped = GRP >= 2 && GRP <= FWD_MAX_GROUP && pos + 1 >= 64;   // the reference's choice (c/src/forward.c:740-744)

  for (int l = 0; l < a.n_layer && ok; ++l) {
    const FwdLayer &Ly = a.layers[l];
    const uint32_t par = static_cast<uint32_t>(l & 1);
    const size_t cache_l = static_cast<size_t>(l) * a.ctx * a.n_kvw;
    trace_stamp(a.trace, 0);
    // the attention head's inputs that do not depend on this layer's activations, into its scratch while phase A runs:
    // the position's rotary row and the QK-norm weights
    if (c < a.n_head && warp == 0 && lane < 3) {
      const bool qkn = a.qk_mode != 0;
      if (lane == 0) {
        mbar_arrive_expect_tx(abar, static_cast<uint32_t>(hd) * 4u * (qkn ? 3u : 1u));
        s_flag[4] = l;
      }
      __syncwarp(7u);
      fence_proxy_async();   // the generic accesses of the scratch (the previous layer's down rows) come first
      float *pre_f = reinterpret_cast<float *>(dslots) + hd;   // rope row, qn, kn (the head's scratch layout below)
      if (lane == 0) bulk_copy_g2s(pre_f, a.rope_cs + static_cast<size_t>(pos) * hd, hd * 4u, abar);
      else if (qkn)
        bulk_copy_g2s(pre_f + lane * hd, lane == 1 ? (a.qk_mode == 1 ? Ly.qn + static_cast<size_t>(c) * hd : Ly.qn)
                                                   : (a.qk_mode == 1 ? Ly.kn + static_cast<size_t>(c / GRP) * hd : Ly.kn), hd * 4u, abar);
    }
    // ---- A: attention input; this CTA's rows of [wq; wk; wv] --------------------------------------------------------
    rmsnorm_to_smem(a.x, Ly.attn_norm, xn, E, a.eps, s_red);
    quant_smem(xn, E, xq_qs, xq_d, xq_bs, warp, NW, lane);
    if (!mbar_wait_bounded(dbar, par)) set_error(&st->err, ERR_WAIT_COPY);
    __syncthreads();
    if (tid == 0) s_flag[5] = 0;
    trace_stamp(a.trace, 14);
    {
      const FwdMat mats[3] = {Ly.wq, Ly.wk, Ly.wv};
      float *outs[3] = {a.qkv + dr0[0], a.qkv + nq + dr0[1], a.qkv + nq + nk + dr0[2]};
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const uint8_t *rows = slots + dense_offset(Ly, dr0, dr1, q) + lo16(mats[q].p + static_cast<size_t>(dr0[q]) * mats[q].rb);
        gemv_rows(mats[q].type, rows, mats[q].rb, nb, dr1[q] - dr0[q], xq_qs, xq_d, xq_bs, outs[q], 0, 0.f);
      }
    }
    trace_stamp(a.trace, 1);
    if (!(ok = grid.sync())) break;
    trace_stamp(a.trace, 2);

    // ---- B: attention, one CTA per query head, no exchange between CTAs -----------------------------------------------------
    // CTA c takes query head c (and c + G, ...): its query and its key/value head's new key and value (QK-norm, rotation,
    // half rounding), the new pair stored by the group's first head; scores against every cached position and the new key
    // (the reference's dotf_h: eight running sums, two threads per position); then, as the reference chooses
    // (c/src/forward.c:740-757): plain: the maximum, e_t = expf(s_t - max), their sum in position order, the values added
    // in position order with weight e_t / sum; grouped: per 256-position chunk its maximum m, e_t = expf(s_t - m), their
    // sum l and the values added with weight e_t, in position order, then the chunks merged (c/src/forward.c:719-737).
    {
      const float *qg = a.qkv, *kg = a.qkv + nq, *vg = a.qkv + nq + nk;
      float *qf = reinterpret_cast<float *>(dslots);                       // [hd] the query
      float *rope_s = qf + hd;                                             // [hd] the position's rotary row (prefetched)
      float *qnw = rope_s + hd, *knw = qnw + hd;                           // [hd] each: the QK-norm weights (prefetched)
      __half *knew = reinterpret_cast<__half *>(knw + hd);                 // [hd] the new key, rounded to half
      __half *vnew = knew + hd;                                            // [hd] the new value
      __half *kvst = vnew + hd;                                            // [FWD_ATT_BLOCK][hd + 8] staged keys or values
      float *scs = reinterpret_cast<float *>(kvst + FWD_ATT_BLOCK * (hd + 8));   // [a chunk] scores, then weights
      float *part = scs + (grouped ? FWD_ATT_CHUNK : ((pos + 1 + 3) & ~3));     // per chunk: maximum, sum, [hd] value sums
      float *s_wmax = s_wt;                                                // [NW] (s_wt is written in the MoE phase)
      for (int h = c; h < a.n_head; h += G) {
        const int g = h / GRP, j = h - g * GRP;
        const bool pre = h == c;   // the first head's rotary row and norm weights are prefetched
        float qscale = 1.f, kscale = 1.f;
        __syncthreads();   // the scratch of the previous head
        if (pre && !mbar_wait_bounded(abar, par)) set_error(&st->err, ERR_WAIT_COPY);
        if (a.qk_mode == 1) {   // QK-norm over the whole query and the whole key (olmoe): their scales
          double sq = 0.0, sk = 0.0;
          for (int i = tid; i < nq; i += FWD_THREADS) { const double v = __ldcg(qg + i); sq += v * v; }
          for (int i = tid; i < nk; i += FWD_THREADS) { const double v = __ldcg(kg + i); sk += v * v; }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) { sq += __shfl_xor_sync(FULL, sq, o); sk += __shfl_xor_sync(FULL, sk, o); }
          if (lane == 0) { s_red[warp] = sq; reinterpret_cast<double *>(terms)[warp] = sk; }
          __syncthreads();
          double tq = 0.0, tk = 0.0;
          for (int k = 0; k < NW; ++k) { tq += s_red[k]; tk += reinterpret_cast<double *>(terms)[k]; }
          qscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tq / nq), a.eps)));
          kscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tk / nk), a.eps)));
        }
        if (warp < 2) {   // warp 0: the query head; warp 1: the key head (and the value)
          const bool isk = warp == 1;
          const float *src = isk ? kg + g * hd : qg + h * hd;
          float v[EPL], vv[EPL];   // the query or the new key; the new value (warp 1), loaded together
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            v[e] = __ldcg(src + lane + 32 * e);
            vv[e] = isk ? __ldcg(vg + g * hd + lane + 32 * e) : 0.f;
          }
          if (a.qk_mode == 2) {   // per head, one shared weight
            double ss = 0.0;
#pragma unroll
            for (int e = 0; e < EPL; ++e) ss += static_cast<double>(v[e]) * v[e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
            const float s1 = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(ss / hd), a.eps)));
            const float *w = pre ? (isk ? knw : qnw) : isk ? Ly.kn : Ly.qn;
#pragma unroll
            for (int e = 0; e < EPL; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], s1), w[lane + 32 * e]);
          } else if (a.qk_mode == 1) {
            const float s1 = isk ? kscale : qscale;
            const float *w = pre ? (isk ? knw : qnw) : isk ? Ly.kn + g * hd : Ly.qn + h * hd;
#pragma unroll
            for (int e = 0; e < EPL; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], s1), w[lane + 32 * e]);
          }
          rope_warp<EPL>(v, pre ? rope_s : a.rope_cs + static_cast<size_t>(pos) * hd, a.rope_pairs != 0);
          if (isk) {
            __half *kd = a.kc + cache_l + static_cast<size_t>(pos) * nk + g * hd;
            __half *vd = a.vc + cache_l + static_cast<size_t>(pos) * nk + g * hd;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
              const __half kh = __float2half_rn(v[e]), vh = __float2half_rn(vv[e]);
              knew[lane + 32 * e] = kh;
              vnew[lane + 32 * e] = vh;
              if (j == 0) { kd[lane + 32 * e] = kh; vd[lane + 32 * e] = vh; }   // kv_put (c/src/forward.c:563-565)
            }
          } else {
#pragma unroll
            for (int e = 0; e < EPL; ++e) qf[lane + 32 * e] = v[e];
          }
        }
        __syncthreads();
        // keys and values pass through shared memory FWD_ATT_BLOCK positions at a time, rows padded by 16 bytes so that
        // consecutive positions (the scores) or consecutive dimensions (the values) fall in different banks
        const __half *kb = a.kc + cache_l + g * hd, *vb = a.vc + cache_l + g * hd;
        const int KS = hd + 8, n = pos + 1;
        auto stage = [&](const __half *base, const __half *fresh, int b0, int cnt) {
          __syncthreads();   // the previous block is consumed
          for (int i = tid; i < cnt * (hd / 8); i += FWD_THREADS) {
            const int t = i / (hd / 8), q = i - t * (hd / 8);
            const uint4 v = b0 + t == pos ? reinterpret_cast<const uint4 *>(fresh)[q]
                                          : __ldcg(reinterpret_cast<const uint4 *>(base + static_cast<size_t>(b0 + t) * nk) + q);
            *reinterpret_cast<uint4 *>(kvst + t * KS + 8 * q) = v;
          }
          __syncthreads();
        };
        // chunk by chunk (grouped: 256 positions; plain: one chunk of every position): scores, one thread per position, the
        // reference's eight running sums combined ((0+1)+(2+3))+((4+5)+(6+7)); the chunk's maximum, e_t, their sum in
        // position order (plain: then e_t / sum); the values in position order, one chain per dimension (thread d)
        const int nchk = grouped ? nchunk : 1, clen = grouped ? FWD_ATT_CHUNK : n;
        for (int ch = 0; ch < nchk; ++ch) {
          const int t0 = ch * clen, t1 = min(n, t0 + clen), m = t1 - t0;
          for (int b0 = t0; b0 < t1; b0 += FWD_ATT_BLOCK) {
            const int cnt = min(FWD_ATT_BLOCK, t1 - b0);
            stage(kb, knew, b0, cnt);
            if (tid < cnt) {
              const __half *kr = kvst + tid * KS;
              float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int i = 0; i < hd; i += 8) {
                const uint4 kk = *reinterpret_cast<const uint4 *>(kr + i);
                const __half2 *k2 = reinterpret_cast<const __half2 *>(&kk);
                const float4 q0 = *reinterpret_cast<const float4 *>(qf + i), q1 = *reinterpret_cast<const float4 *>(qf + i + 4);
                const float2 k01 = __half22float2(k2[0]), k23 = __half22float2(k2[1]), k45 = __half22float2(k2[2]), k67 = __half22float2(k2[3]);
                s8[0] = __fadd_rn(s8[0], __fmul_rn(q0.x, k01.x));
                s8[1] = __fadd_rn(s8[1], __fmul_rn(q0.y, k01.y));
                s8[2] = __fadd_rn(s8[2], __fmul_rn(q0.z, k23.x));
                s8[3] = __fadd_rn(s8[3], __fmul_rn(q0.w, k23.y));
                s8[4] = __fadd_rn(s8[4], __fmul_rn(q1.x, k45.x));
                s8[5] = __fadd_rn(s8[5], __fmul_rn(q1.y, k45.y));
                s8[6] = __fadd_rn(s8[6], __fmul_rn(q1.z, k67.x));
                s8[7] = __fadd_rn(s8[7], __fmul_rn(q1.w, k67.y));
              }
              const float d = __fadd_rn(__fadd_rn(__fadd_rn(s8[0], s8[1]), __fadd_rn(s8[2], s8[3])),
                                        __fadd_rn(__fadd_rn(s8[4], s8[5]), __fadd_rn(s8[6], s8[7])));
              scs[b0 - t0 + tid] = __fmul_rn(d, a.attn_scale);
            }
          }
          __syncthreads();
          trace_stamp(a.trace, 15);
          float mx = -INFINITY;   // the chunk's maximum: every thread's share, each warp's, then the warps'
          for (int t = tid; t < m; t += FWD_THREADS) mx = fmaxf(mx, scs[t]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
          if (lane == 0) s_wmax[warp] = mx;
          __syncthreads();
          mx = s_wmax[0];
          for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s_wmax[w]);
          for (int t = tid; t < m; t += FWD_THREADS) scs[t] = exp_cr(__fsub_rn(scs[t], mx));
          __syncthreads();
          if (tid == 0) {   // the sum in position order
            float l = 0.f;
            for (int t = 0; t < m; ++t) l = __fadd_rn(l, scs[t]);
            part[ch * (2 + hd)] = mx;
            part[ch * (2 + hd) + 1] = l;
          }
          trace_stamp(a.trace, 16);
          if (!grouped) {   // plain: p_t = e_t / sum
            __syncthreads();
            const float sum = part[1];
            for (int t = tid; t < m; t += FWD_THREADS) scs[t] = __fdiv_rn(scs[t], sum);
          }
          float o = 0.f;
          for (int b0 = t0; b0 < t1; b0 += FWD_ATT_BLOCK) {
            const int cnt = min(FWD_ATT_BLOCK, t1 - b0);
            stage(vb, vnew, b0, cnt);
            if (tid < hd)
              for (int t = 0; t < cnt; ++t) o = __fadd_rn(o, __fmul_rn(scs[b0 - t0 + t], __half2float(kvst[t * KS + tid])));
          }
          if (tid < hd) {
            if (!grouped) __stcg(a.att + h * hd + tid, o);
            else part[ch * (2 + hd) + 2 + tid] = o;
          }
          __syncthreads();   // scs and the staging buffer are reused by the next chunk
        }
        if (grouped) {
          __syncthreads();
          for (int d = tid; d < hd; d += FWD_THREADS) {
            if (nchk == 1) {   // the merge of one chunk: weight expf(0) = 1, so o * (1 / l)
              __stcg(a.att + h * hd + d, __fmul_rn(part[2 + d], __fdiv_rn(1.0f, part[1])));
            } else {
              float M = -INFINITY;
              for (int ch = 0; ch < nchk; ++ch) M = fmaxf(M, part[ch * (2 + hd)]);
              float L = 0.f, o = 0.f;
              for (int ch = 0; ch < nchk; ++ch) {
                const float *pp = part + ch * (2 + hd);
                const float w = exp_cr(__fsub_rn(pp[0], M));
                L = __fadd_rn(L, __fmul_rn(w, pp[1]));
                o = __fadd_rn(o, __fmul_rn(w, pp[2 + d]));
              }
              __stcg(a.att + h * hd + d, __fmul_rn(o, __fdiv_rn(1.0f, L)));
            }
          }
        }
        trace_stamp(a.trace, 17);
      }
    }
    if (!(ok = grid.sync())) break;
    trace_stamp(a.trace, 4);

    // ---- C: attention output: x += resid * wo att, this CTA's rows ------------------------------------------------------
    quant_global(a.att, nq / 256, xq_qs, xq_d, xq_bs, warp, NW, lane);
    __syncthreads();
    gemv_rows(Ly.wo.type, slots + dense_offset(Ly, dr0, dr1, 3) + lo16(Ly.wo.p + static_cast<size_t>(i0) * Ly.wo.rb), Ly.wo.rb, nq / 256, nd,
              xq_qs, xq_d, xq_bs, a.x + i0, 1, a.resid_scale);
    trace_stamp(a.trace, 5);
    if (!(ok = grid.sync())) break;
    trace_stamp(a.trace, 6);

    // ---- D: mixture of experts -------------------------------------------------------------------------------------------
    rmsnorm_to_smem(a.x, Ly.ffn_norm, xn, E, a.eps, s_red);
    for (int i = i0 + tid; i < i1; i += FWD_THREADS) xr[i - i0] = __ldcg(a.x + i);
    if (s_flag[1] && !mbar_wait_bounded(rbar, par)) set_error(&st->err, ERR_WAIT_COPY);
    for (int m = 0; m < nre; ++m)   // the router products, laid out for the strided sums
      for (int i = tid; i < E; i += FWD_THREADS) rprod[(m * 8 + (i & 7)) * RS + (i >> 3)] = __fmul_rn(rrows[m * E + i], xn[i]);
    __syncthreads();
    if (tid == 0) {   // the next layer's router rows, while this one's are consumed from the products
      s_flag[1] = 0;
      if (nre > 0 && l + 1 < a.n_layer) {
        s_flag[3] = (l + 1) & 1;
        fence_proxy_async();   // the generic reads of rrows before the bulk copy's writes
        mbar_arrive_expect_tx(rbar, static_cast<uint32_t>(nre) * E * 4u);
        for (int m = 0; m < nre; ++m)
          bulk_copy_g2s_hint(rrows + static_cast<size_t>(m) * E, a.layers[l + 1].router + static_cast<size_t>(c + m * G) * E, E * 4u, rbar, l2_evict_first());
        s_flag[1] = 1;
      }
    }
    if (warp == RW) {
      if (nre > 0) {
        const int grp = lane >> 3, l8 = lane & 7;
        for (int m0 = 0; m0 < nre; m0 += 4) {
          const int m = m0 + grp;
          float s = 0.f;
          if (m < nre) {
            const float4 *p4 = reinterpret_cast<const float4 *>(rprod + (m * 8 + l8) * RS);
            for (int q = 0; q < E / 32; q += 4) {
              float4 v[4];
#pragma unroll
              for (int t = 0; t < 4; ++t) v[t] = p4[q + t];
#pragma unroll
              for (int t = 0; t < 4; ++t) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[t].x), v[t].y), v[t].z), v[t].w);
            }
          }
          float p8[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) p8[k] = __shfl_sync(FULL, s, (lane & ~7) + k);
          if (m < nre && l8 == 0)
            a.rlogits[c + m * G] = __fadd_rn(__fadd_rn(__fadd_rn(p8[0], p8[1]), __fadd_rn(p8[2], p8[3])),
                                             __fadd_rn(__fadd_rn(p8[4], p8[5]), __fadd_rn(p8[6], p8[7])));
        }
        __syncwarp();
        if (lane == 0) red_release_add(&st->sync[1], static_cast<uint32_t>(nre));
        if (lane == 0) trace_stamp_here(a.trace, 19);
      }
    } else {
      quant_smem(xn, E, xq_qs, xq_d, xq_bs, warp, RW, lane);
    }
    trace_stamp(a.trace, 7);
    // softmax (c/src/forward.c:954-958) over FWD_MAX_NE threads, one expert each: the maximum, e = expf(l - max), the sum
    // in double (each warp's 32 experts by a shuffle tree, then the warps in order), p = (float)(e / sum)
    if (tid == 0) {
      const uint32_t target = static_cast<uint32_t>(NE) * static_cast<uint32_t>(l + 1);
      bool got = false;
#pragma unroll 1
      for (uint32_t i = 0; i < SPIN_LIMIT; ++i) {
        if (ld_acquire(&st->sync[1]) >= target) { got = true; break; }
        if ((i & 127) == 127 && ld_volatile(&st->err)) break;
        if (i > 4096) __nanosleep(64);
      }
      if (!got) set_error(&st->err, ERR_WAIT_ROUTER);
      s_flag[2] = got;
      trace_stamp_here(a.trace, 20);
    }
    __syncthreads();
    if (!s_flag[2]) { ok = false; break; }
    // routing (c/src/forward.c:954-984) with this CTA's share of the experts sent out on the logit order at once: softmax is
    // monotone, so that is the probability order except where two different logits round to the same probability. The
    // softmax (double sum), the probability order and the weights follow while the copies fly; a slot whose expert turns
    // out not to be chosen (a probability tie at rank K) fetches the missing one on its mbarrier's next phase. Slot k holds
    // expert s_spec[k]; the expert of rank r sits in slot s_slot[r].
    constexpr int SW = FWD_MAX_NE / 32;   // softmax warps, one expert per thread
    const float lgv = tid < NE ? __ldcg(a.rlogits + tid) : -INFINITY;
    float mx = lgv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0 && warp < SW) s_wt[warp] = mx;   // s_wt is written after the ranking
    // NaN ranks as -inf here, so the ranks by logit are a permutation and every slot gets one expert (a NaN routing then
    // fails in the probability check below, with every copy accounted for)
    if (tid < FWD_MAX_NE) s_lg[tid] = lgv == lgv ? lgv : -INFINITY;
    if (tid <= FWD_MAX_K) s_spec[tid] = -1;
    if (tid < FWD_MAX_K) s_fix[tid] = 0;
    __syncthreads();
    mx = s_wt[0];
#pragma unroll
    for (int w = 1; w < SW; ++w) mx = fmaxf(mx, s_wt[w]);
    // rank of expert tid / 4 = experts ahead of it in the reference's arg-max order (ties to the lower id), counted by four
    // threads over every fourth float4 of the values each (v padded with `pad`, below every value, to a multiple of 4)
    auto rank4 = [&](const float *v, float pad) -> int {
      const int e = tid >> 2, part = tid & 3, n4 = (NE + 3) / 4;
      const float pe = e < NE ? v[e] : 0.f;
      const float4 *p4 = reinterpret_cast<const float4 *>(v);
      float4 q[8];   // n4 <= 32 (NE <= 128): every load in flight before the first comparison
#pragma unroll
      for (int u = 0; u < 8; ++u) q[u] = 4 * u + part < n4 ? p4[4 * u + part] : make_float4(pad, pad, pad, pad);
      int rank = 0;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int f = 4 * (4 * u + part);
        rank += (q[u].x > pe || (q[u].x == pe && f < e)) + (q[u].y > pe || (q[u].y == pe && f + 1 < e)) +
                (q[u].z > pe || (q[u].z == pe && f + 2 < e)) + (q[u].w > pe || (q[u].w == pe && f + 3 < e));
      }
      rank += __shfl_xor_sync(FULL, rank, 1);
      rank += __shfl_xor_sync(FULL, rank, 2);
      return rank;
    };
    // one thread: expert e's share for this CTA into slot k (gate and up rows into the slots, down rows into the dslots),
    // on the slot's mbarrier; s_cnt[k] counts the slot's phases (its parity is the one to wait for)
    auto issue = [&](int k, int e) {
      uint8_t *gs = slots + static_cast<size_t>(k) * a.slot_bytes, *ds = dslots + static_cast<size_t>(k) * a.dslot_bytes;
      const size_t ex = static_cast<size_t>(e);
      const uint8_t *src[3] = {Ly.gate + ex * Ly.gate_slab + static_cast<size_t>(j0) * a.grb,
                               Ly.up + ex * Ly.up_slab + static_cast<size_t>(j0) * a.grb,
                               Ly.down + ex * Ly.down_slab + static_cast<size_t>(i0) * a.drb};
      uint8_t *dst[3] = {gs, gs + a.gseg, ds};
      const uint32_t len[3] = {static_cast<uint32_t>(ngu) * a.grb, static_cast<uint32_t>(ngu) * a.grb, static_cast<uint32_t>(nd) * a.drb};
      uint32_t n16[3], total = 0;
      for (int q = 0; q < 3; ++q) { n16[q] = len[q] ? (lo16(src[q]) + len[q] + 15u) & ~15u : 0u; total += n16[q]; }
      fence_proxy_async();   // the generic accesses of these buffers (attention scratch, dense rows) come first
      mbar_arrive_expect_tx(&bars[k], total);
      for (int q = 0; q < 3; ++q)
        if (n16[q]) bulk_copy_g2s_hint(dst[q], src[q] - lo16(src[q]), n16[q], &bars[k], l2_evict_first());
      s_cnt[k] += 1;
    };
    {
      int rank = rank4(s_lg, -INFINITY);
      if (a.force_miss && K < NE) rank = rank == K - 1 ? K : rank == K ? K - 1 : rank;   // test hook: ranks K - 1 and K swap
      if ((tid >> 2) < NE && (tid & 3) == 0 && rank <= K) {
        s_spec[rank] = tid >> 2;
        if (rank < K) issue(rank, tid >> 2);
      }
    }
    trace_stamp(a.trace, 21);
    {
      const float ev = tid < NE ? exp_cr(__fsub_rn(lgv, mx)) : 0.f;
      double part = static_cast<double>(ev);   // each warp's 32 experts by a shuffle tree, then the warps in order
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(FULL, part, o);
      if (lane == 0 && warp < SW) s_red[warp] = part;
      __syncthreads();
      double tot = 0.0;
#pragma unroll
      for (int w = 0; w < SW; ++w) tot += s_red[w];
      if (tid < ((NE + 3) & ~3)) probs[tid] = tid < NE ? __double2float_rn(__ddiv_rn(static_cast<double>(ev), tot)) : -1.0f;
    }
    __syncthreads();
    trace_stamp(a.trace, 22);
    if (warp == 0) {   // strictly falling probabilities along the logit order through rank K: that order is the reference's
      const int n = K < NE ? K + 1 : K;
      const int se = lane < n ? s_spec[lane] : 0;
      const float pl = lane < n && se >= 0 ? probs[se] : 0.f;
      const float pn = __shfl_down_sync(FULL, pl, 1);
      const bool strict = __all_sync(FULL, se >= 0 && (lane + 1 >= n || pl > pn));
      if (strict && lane < K) {
        s_sel[lane] = se;
        s_wt[lane] = pl;
        s_slot[lane] = lane;
      }
      if (lane == 0) s_flag[7] = strict ? 0 : 1;
    }
    __syncthreads();
    trace_stamp(a.trace, 27);
    if (s_flag[7]) {   // the full probability order (c/src/forward.c:975-980), then every chosen expert into a slot
      const int e = tid >> 2;
      const int rank = rank4(probs, -1.0f);
      if (e < NE && (tid & 3) == 0 && rank < K) { s_sel[rank] = e; s_wt[rank] = probs[e]; }
      __syncthreads();
      const int tk0 = tid < K ? s_sel[tid] : 0;
      if (warp == 0 && __any_sync(FULL, tk0 < 0 || tk0 >= NE)) {   // logits that do not order (NaN): no expert to fetch
        if (lane == 0) set_error(&st->err, ERR_BAD_EXPERT);
      } else if (warp == 0) {
        // a slot holding an expert outside the top k takes a missing one: the missing rank's position among the missing
        // ranks pairs it with the orphan slot at the same position
        int gk = -1;
        const int tk = lane < K ? s_sel[lane] : -2;
        for (int h = 0; h < K; ++h) gk = s_spec[h] == tk ? h : gk;
        const int sg = lane < K ? s_spec[lane] : -2;
        bool in = false;
        for (int k = 0; k < K; ++k) in |= s_sel[k] == sg;
        const uint32_t orphan = __ballot_sync(FULL, lane < K && !in), missing = __ballot_sync(FULL, lane < K && gk < 0);
        if (lane < K && gk < 0) {
          const int at = __popc(missing & ((1u << lane) - 1u));
          uint32_t o = orphan;
          for (int t = 0; t < at && o; ++t) o &= o - 1u;
          gk = o ? __ffs(o) - 1 : -1;
          if (gk >= 0) s_fix[gk] = tk + 1;
        }
        if (lane < K) s_slot[lane] = gk >= 0 ? gk : 0;
        if (lane < K && (gk < 0 || tk < 0)) set_error(&st->err, ERR_BAD_EXPERT);   // two sets of K: cannot happen
      }
      __syncthreads();
      trace_stamp(a.trace, 26);
      if (warp < K && lane == 0 && s_fix[warp]) {   // the wrong copies land first; then the right expert's
        const int k = warp;
        if (mbar_wait_bounded(&bars[k], static_cast<uint32_t>((s_cnt[k] - 1) & 1))) {
          s_spec[k] = s_fix[k] - 1;
          issue(k, s_spec[k]);
        } else {
          set_error(&st->err, ERR_WAIT_COPY);
        }
      }
      __syncthreads();
    }
    if (tid < K) {   // renormalisation (c/src/forward.c:984)
      float w = s_wt[tid];
      if (a.norm_topk) {
        float z = 0.f;
        for (int k = 0; k < K; ++k) z = __fadd_rn(z, s_wt[k]);
        if (z > 0.f) w = __fdiv_rn(w, z);
      }
      s_wn[tid] = w;
      if (c == 0) {
        a.route_sel[l * K + tid] = s_sel[tid];
        a.route_wt[l * K + tid] = w;
      }
    }
    __syncthreads();   // s_wn, s_slot and s_spec for every thread
    trace_stamp(a.trace, 8);
    auto gu_src = [&](int k, int q) -> const uint8_t * {   // slot k's gate (q 0) or up (q 1) rows in global memory
      const size_t e = static_cast<size_t>(s_spec[k]);
      return q == 0 ? Ly.gate + e * Ly.gate_slab + static_cast<size_t>(j0) * a.grb : Ly.up + e * Ly.up_slab + static_cast<size_t>(j0) * a.grb;
    };
    auto dn_src = [&](int k) -> const uint8_t * { return Ly.down + static_cast<size_t>(s_spec[k]) * Ly.down_slab + static_cast<size_t>(i0) * a.drb; };
    // gate and up rows: a group of lanes per (expert, row), one lane per block
    {
      const int GL = lanes_for(nb);
      const int lg = lane & (GL - 1), gpw = 32 / GL, ngroups = NW * gpw, gid = warp * gpw + lane / GL;
      const int tasks = K * ngu, base = lane - lg;
      const bool has_blk = lg < nb;
      int waited = -1;
      for (int t0 = 0; t0 < tasks; t0 += ngroups) {
        const int t = t0 + gid;
        const bool valid = t < tasks;
        const int k = valid ? t / ngu : 0, j = valid ? t - k * ngu : 0;
        float tg = 0.f, tu = 0.f;
        if (valid) {
          while (waited < k) {
            ++waited;
            if (!mbar_wait_bounded(&bars[waited], static_cast<uint32_t>((s_cnt[waited] - 1) & 1))) set_error(&st->err, ERR_WAIT_COPY);
          }
          if (has_blk) {
            const uint8_t *gs = slots + static_cast<size_t>(k) * a.slot_bytes;
            tg = blk_dot(Ly.gate_type, gs + lo16(gu_src(k, 0)) + static_cast<uint32_t>(j) * a.grb, lg, xq_qs, xq_bs, xq_d, lg);
            tu = blk_dot(Ly.gate_type, gs + a.gseg + lo16(gu_src(k, 1)) + static_cast<uint32_t>(j) * a.grb, lg, xq_qs, xq_bs, xq_d, lg);
          }
        }
        float sg = 0.f, su = 0.f;
        for (int b = 0; b < nb; ++b) {
          sg = __fadd_rn(sg, __shfl_sync(FULL, tg, base + b));
          su = __fadd_rn(su, __shfl_sync(FULL, tu, base + b));
        }
        if (valid && lg == 0) __stcg(a.hg + static_cast<size_t>(k) * FF + j0 + j, swiglu(sg, su));
      }
    }
    trace_stamp(a.trace, 9);
    if (!(ok = grid.sync())) break;
    trace_stamp(a.trace, 10);
    if (tid == 0 && l + 1 < a.n_layer) {   // the next layer's dense rows into the slots, whose gate/up rows are consumed
      issue_dense(a.layers[l + 1], slots, dbar, dr0, dr1);
      s_flag[5] = 1;
      s_flag[6] = (l + 1) & 1;
    }
    // every expert's hg as Q8_K blocks; this CTA's down rows; the combine in rank order and the residual
    quant_global(a.hg, K * FF / 256, hq_qs, hq_d, hq_bs, warp, NW, lane);
    trace_stamp(a.trace, 23);
    for (int k = 0; k < K; ++k)
      if (!mbar_wait_bounded(&bars[k], static_cast<uint32_t>((s_cnt[k] - 1) & 1))) set_error(&st->err, ERR_WAIT_COPY);
    __syncthreads();
    trace_stamp(a.trace, 24);
    {   // down rows: a group of lanes per (expert, block), one row per lane, so the group's activation reads are broadcasts
      const int C = K * nbd, LP = nd > 16 ? 32 : 16, ppw = 32 / LP, lp = lane & (LP - 1);
      for (int p = warp * ppw + lane / LP; p < C; p += NW * ppw) {
        const int k = p / nbd, blk = p - k * nbd;
        const uint8_t *drows = dslots + static_cast<size_t>(k) * a.dslot_bytes + lo16(dn_src(k));
        for (int r = lp; r < nd; r += LP)   // p = k * nbd + blk: the block's index in the Q8_K of every expert's hg
          terms[(r * K + k) * nbd + blk] = blk_dot(Ly.down_type, drows + static_cast<size_t>(r) * a.drb, blk, hq_qs, hq_bs, hq_d, p);
      }
    }
    __syncthreads();
    trace_stamp(a.trace, 25);
    {   // wt * hd per (row, rank), hd the block terms in block order; then per row their sum in rank order, the residual
      float *wprod = rprod;   // [nd][K] (the router products are done with)
      for (int q = tid; q < nd * K; q += FWD_THREADS) {   // q = row * K + rank; the terms are by slot
        const int r = q / K, k = q - r * K;
        const float *tq = terms + (r * K + s_slot[k]) * nbd;
        float h = 0.f;
#pragma unroll 4
        for (int b = 0; b < nbd; ++b) h = __fadd_rn(h, tq[b]);
        wprod[q] = __fmul_rn(s_wn[k], h);
      }
      __syncthreads();
      for (int r = tid; r < nd; r += FWD_THREADS) {
        float moe = 0.f;
#pragma unroll 8
        for (int k = 0; k < K; ++k) moe = __fadd_rn(moe, wprod[r * K + k]);
        a.x[i0 + r] = __fadd_rn(xr[r], __fmul_rn(a.resid_scale, moe));
      }
    }
    trace_stamp(a.trace, 11);
    if (!(ok = grid.sync())) break;
  }

  // ---- output norm, this CTA's rows of the output matrix, arg-max ------------------------------------------------------------
  if (ok) {
    trace_stamp(a.trace, 12);
    rmsnorm_to_smem(a.x, a.out_norm, xn, E, a.eps, s_red);
    quant_smem(xn, E, xq_qs, xq_d, xq_bs, warp, NW, lane);
    __syncthreads();
    const int v0 = static_cast<int>(static_cast<uint64_t>(a.vocab) * uc / uG), v1 = static_cast<int>(static_cast<uint64_t>(a.vocab) * (uc + 1) / uG);
    const int nst = (v1 - v0 + HEAD_ROWS - 1) / HEAD_ROWS;
    // a stage holds HEAD_ROWS rows copied from the 16-byte boundary at or below their start (rows of a Q6_K matrix may
    // start anywhere), so it is 32 bytes longer than the rows and they begin lo16 bytes into it; the stages use the
    // slots and dslots together. Two stages are computed at a time (half the lane groups each), HEAD_STAGES in flight.
    const uint32_t rb = a.output.rb, stage_bytes = (HEAD_ROWS * rb + 32 + 15) & ~15u;
    auto stage_src = [&](int s) { return a.output.p + static_cast<size_t>(v0 + s * HEAD_ROWS) * rb; };
    auto issue = [&](int s) {
      const int cnt = min(HEAD_ROWS, v1 - (v0 + s * HEAD_ROWS));
      const uint8_t *src = stage_src(s);
      const uint32_t n16 = (lo16(src) + static_cast<uint32_t>(cnt) * rb + 15u) & ~15u;
      uint64_t *b = &hb[s % HEAD_STAGES];
      fence_proxy_async();
      mbar_arrive_expect_tx(b, n16);
      bulk_copy_g2s_hint(slots + static_cast<size_t>(s % HEAD_STAGES) * stage_bytes, src - lo16(src), n16, b, l2_evict_first());
    };
    if (tid == 0)
      for (int s = 0; s < min(nst, HEAD_STAGES); ++s) issue(s);
    const int GL = lanes_for(nb), lg = lane & (GL - 1), gpw = 32 / GL, ngroups = NW * gpw, gid = warp * gpw + lane / GL, base = lane - lg;
    const int half = ngroups / 2, side = gid / half, hg = gid - side * half;   // which of the two stages, and the group in it
    const bool has_blk = lg < nb;
    unsigned long long best = 0;
    for (int s0 = 0; s0 < nst; s0 += 2) {
      const int s = s0 + side;
      const bool live = s < nst;
      if (live && !mbar_wait_bounded(&hb[s % HEAD_STAGES], static_cast<uint32_t>((s / HEAD_STAGES) & 1))) set_error(&st->err, ERR_WAIT_COPY);
      const int r0 = v0 + s * HEAD_ROWS, cnt = live ? min(HEAD_ROWS, v1 - r0) : 0;
      const uint8_t *buf = slots + static_cast<size_t>(s % HEAD_STAGES) * stage_bytes + (live ? lo16(stage_src(s)) : 0u);
      for (int q0 = 0; q0 < HEAD_ROWS; q0 += half) {   // the same trip count in every warp
        const int q = q0 + hg;
        const bool valid = q < cnt;
        float t = 0.f;
        if (valid && has_blk) t = blk_dot_fast(a.output.type, buf + static_cast<size_t>(q) * rb, lg, xq_qs, xq_bs, xq_d, lg);
        float sum = 0.f;
        for (int b = 0; b < nb; ++b) sum = __fadd_rn(sum, __shfl_sync(FULL, t, base + b));
        if (valid && lg == 0) {
          const float v = a.logit_scale != 1.0f ? __fdiv_rn(sum, a.logit_scale) : sum;
          __stcg(a.logits + r0 + q, v);
          if (v == v) best = max(best, argmax_key(v, r0 + q));
        }
      }
      __syncthreads();   // both buffers are free again
      if (tid == 0) {
        if (s0 + HEAD_STAGES < nst) issue(s0 + HEAD_STAGES);
        if (s0 + 1 + HEAD_STAGES < nst) issue(s0 + 1 + HEAD_STAGES);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(FULL, best, o));
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < NW; ++w) best = max(best, s_best[w]);
      atomicMax(&st->best, best);
    }
    trace_stamp(a.trace, 13);
  }

  // ---- exit: copies in flight land first; the last CTA out advances the sequence and resets the counters ----------------------
  __syncthreads();
  if (tid == 0) {
    if (s_flag[1]) mbar_wait_bounded(rbar, static_cast<uint32_t>(s_flag[3]));   // an unconsumed router copy
    if (s_flag[5]) mbar_wait_bounded(dbar, static_cast<uint32_t>(s_flag[6]));   // an unconsumed dense copy
    if (s_flag[4] >= 0) mbar_wait_bounded(abar, static_cast<uint32_t>(s_flag[4] & 1));   // the last attention prefetch
    for (int k = 0; k < K; ++k)   // each slot's last copies (waited already unless a wait gave up)
      if (s_cnt[k] > 0) mbar_wait_bounded(&bars[k], static_cast<uint32_t>((s_cnt[k] - 1) & 1));
    __threadfence();
    const uint32_t prev = atomicAdd(&st->sync[2], 1u);
    if (prev == uG - 1) {
      __threadfence();
      if (!ld_volatile(&st->err)) {
        const unsigned long long b = atomicAdd(&st->best, 0ull);
        const int id = static_cast<int>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffull));
        st->next = id;
        a.gen_out[pos] = id;
        if (a.feed) st->token = id;
        st->pos = pos + 1;
      }
      st->best = 0;
      atomicExch(&st->sync[0], 0u);
      atomicExch(&st->sync[1], 0u);
      atomicExch(&st->sync[2], 0u);
      __threadfence();
    }
  }
  trace_time(a.trace, 31);
}

}  // namespace

cudaError_t fwd_allow_smem(int bytes) {
  cudaError_t e = cudaFuncSetAttribute(fwd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fwd_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e;
}

cudaError_t fwd_launch(const FwdArgs &a, int ctas, cudaStream_t stream) {
  void (*fn)(FwdArgs) = a.hd == 64 ? fwd_kernel<2> : a.hd == 128 ? fwd_kernel<4> : a.hd == 256 ? fwd_kernel<8> : nullptr;
  if (!fn) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(FWD_THREADS);
  cfg.dynamicSmemBytes = a.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace clb
