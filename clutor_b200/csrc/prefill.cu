// Per-token kernels of the batched prompt path (run_std, c/src/forward.c:1078-1225): the embedding, rmsnorm + Q8_K,
// QK-norm + rotary embedding + the key/value store, and the plain attention of every (token, head). Every float operation
// the reference rounds is one explicitly rounded operation here, in the reference's order, as in the one-token step.
#include <algorithm>

#include "common.cuh"
#include "decode.cuh"
#include "modelops.cuh"
#include "prefill.cuh"
#include "rowdot.cuh"

namespace clb {
namespace {

constexpr int PT = 256;          // threads of the per-token kernels
constexpr int PNW = PT / 32;
constexpr int AT = 128;          // threads of an attention task

__global__ void __launch_bounds__(PT) embed_kernel(FwdMat emb, const int *tok, int E, float scale, float *X) {
  float *x = X + static_cast<size_t>(blockIdx.x) * E;
  embed_row(emb, tok[blockIdx.x], E, x);
  if (scale != 1.0f)   // c/src/forward.c:1087: x[i] *= embed_scale (each thread scales the elements it wrote)
    for (int i = threadIdx.x; i < E; i += blockDim.x) x[i] = __fmul_rn(x[i], scale);
}

// rmsnorm (double sum of squares: per thread, a shuffle tree, then the warps in order) into shared memory, then Q8_K
__global__ void __launch_bounds__(PT) norm_q8k_kernel(const float *X, int row0, int E, const float *w, float eps, int8_t *qs,
                                                      float *dd, int16_t *bs) {
  __shared__ __align__(16) float xn[4096];
  __shared__ double red[PNW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, b = blockIdx.x;
  const float *x = X + static_cast<size_t>(row0 + b) * E;
  double ss = 0.0;
  for (int i = tid; i < E; i += PT) {
    const float v = x[i];
    ss += static_cast<double>(v) * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  double tot = 0.0;
  for (int k = 0; k < PNW; ++k) tot += red[k];
  const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(__ddiv_rn(tot, static_cast<double>(E))), eps)));
  for (int i = tid; i < E; i += PT) xn[i] = __fmul_rn(__fmul_rn(x[i], s), w[i]);
  __syncthreads();
  q8k_quantize_block(xn, E, qs + static_cast<size_t>(b) * E, dd + static_cast<size_t>(b) * (E / 256),
                     bs + static_cast<size_t>(b) * (E / 16), warp, PNW, lane, false);
}

__global__ void __launch_bounds__(PT) q8k_kernel(const float *src, int cols, int8_t *qs, float *dd, int16_t *bs) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, b = blockIdx.x;
  q8k_quantize_global(src + static_cast<size_t>(b) * cols, cols / 256, qs + static_cast<size_t>(b) * cols,
                      dd + static_cast<size_t>(b) * (cols / 256), bs + static_cast<size_t>(b) * (cols / 16), warp, PNW, lane, false);
  (void)tid;
}

// One token per CTA; a warp per head (query heads, then key heads).
template <int EPL>
__global__ void __launch_bounds__(PT) qk_kernel(const PfQkArgs a) {
  __shared__ double red[2][PNW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, b = blockIdx.x, hd = a.hd;
  const int nq = a.n_head * hd, nk = a.n_kv * hd, pos = a.pos0 + b, GRP = a.n_head / a.n_kv;
  const float *q = a.Q + static_cast<size_t>(b) * nq, *k = a.K + static_cast<size_t>(b) * nk, *v = a.V + static_cast<size_t>(b) * nk;
  float qscale = 1.f, kscale = 1.f;
  if (a.qk_mode == 1) {   // QK-norm over the whole query and the whole key (c/src/forward.c:1106): their scales
    double sq = 0.0, sk = 0.0;
    for (int i = tid; i < nq; i += PT) { const double t = q[i]; sq += t * t; }
    for (int i = tid; i < nk; i += PT) { const double t = k[i]; sk += t * t; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) { sq += __shfl_xor_sync(FULL, sq, o); sk += __shfl_xor_sync(FULL, sk, o); }
    if (lane == 0) { red[0][warp] = sq; red[1][warp] = sk; }
    __syncthreads();
    double tq = 0.0, tk = 0.0;
    for (int w = 0; w < PNW; ++w) { tq += red[0][w]; tk += red[1][w]; }
    qscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tq / nq), a.eps)));
    kscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tk / nk), a.eps)));
  }
  const float *cs = a.rope_cs + static_cast<size_t>(pos) * hd;
  for (int h = warp; h < a.n_head + a.n_kv; h += PNW) {
    const bool isk = h >= a.n_head;
    const int head = isk ? h - a.n_head : h;
    const float *src = (isk ? k : q) + head * hd;
    float x[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) x[e] = src[lane + 32 * e];
    if (a.qk_mode == 2) {   // per head, one weight vector shared by the heads (c/src/forward.c:1105)
      double ss = 0.0;
#pragma unroll
      for (int e = 0; e < EPL; ++e) ss += static_cast<double>(x[e]) * x[e];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
      const float s1 = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(ss / hd), a.eps)));
      const float *w = isk ? a.kn : a.qn;
#pragma unroll
      for (int e = 0; e < EPL; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], s1), w[lane + 32 * e]);
    } else if (a.qk_mode == 1) {
      const float s1 = isk ? kscale : qscale;
      const float *w = (isk ? a.kn : a.qn) + head * hd;
#pragma unroll
      for (int e = 0; e < EPL; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], s1), w[lane + 32 * e]);
    }
    rope_warp<EPL>(x, cs, a.rope_pairs != 0);
    if (isk) {   // kv_put (c/src/forward.c:563-565): the key and the value, rounded to half
      __half *kd = a.kc + static_cast<size_t>(pos) * nk + head * hd, *vd = a.vc + static_cast<size_t>(pos) * nk + head * hd;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        kd[lane + 32 * e] = __float2half_rn(x[e]);
        vd[lane + 32 * e] = __float2half_rn(v[head * hd + lane + 32 * e]);
      }
    } else {
      float *dst = a.Qr + static_cast<size_t>(b) * nq + head * hd;
#pragma unroll
      for (int e = 0; e < EPL; ++e) dst[lane + 32 * e] = x[e];
    }
  }
  (void)GRP;
}

// One (query head, token) per CTA. Shared memory: the query [hd] and the scores [pos + 1].
__global__ void __launch_bounds__(AT) attn_kernel(const PfAttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[AT / 32];
  __shared__ float s_sum;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.x, b = blockIdx.y, hd = a.hd, nq = a.n_head * hd, KW = a.n_kvw;
  const int pos = a.pos0 + b, n = pos + 1, g = h / (a.n_head / a.n_kv);
  float *q = sm, *sc = sm + hd;
  for (int i = tid; i < hd; i += AT) q[i] = a.Qr[static_cast<size_t>(b) * nq + h * hd + i];
  __syncthreads();
  // scores: the reference's dotf_h (c/src/forward.c:492-510), eight running sums combined ((0+1)+(2+3))+((4+5)+(6+7))
  float mx = -INFINITY;
  const __half *kb = a.kc + g * hd;
  for (int t = tid; t < n; t += AT) {
    const __half *kr = kb + static_cast<size_t>(t) * KW;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < hd; i += 8) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(kr + i);
      const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = __half22float2(h2[u]);
        s[2 * u] = __fadd_rn(s[2 * u], __fmul_rn(q[i + 2 * u], f.x));
        s[2 * u + 1] = __fadd_rn(s[2 * u + 1], __fmul_rn(q[i + 2 * u + 1], f.y));
      }
    }
    const float d = __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3])), __fadd_rn(__fadd_rn(s[4], s[5]), __fadd_rn(s[6], s[7])));
    const float v = __fmul_rn(d, a.attn_scale);
    sc[t] = v;
    if (v > mx) mx = v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < AT / 32; ++w) mx = fmaxf(mx, red[w]);
  for (int t = tid; t < n; t += AT) sc[t] = expf_cr(__fsub_rn(sc[t], mx));
  __syncthreads();
  if (tid == 0) {   // the float sum in position order (c/src/forward.c:602-603)
    float sum = 0.f;
    for (int t = 0; t < n; ++t) sum = __fadd_rn(sum, sc[t]);
    s_sum = sum;
  }
  __syncthreads();
  const float sum = s_sum;
  for (int t = tid; t < n; t += AT) sc[t] = __fdiv_rn(sc[t], sum);
  __syncthreads();
  // values: axpy_h (c/src/forward.c:512-521) in position order, one thread per element of the head
  const __half *vb = a.vc + g * hd;
  for (int d = tid; d < hd; d += AT) {
    float o = 0.f;
    int t = 0;
    for (; t + 4 <= n; t += 4) {
      const float v0 = __half2float(vb[static_cast<size_t>(t) * KW + d]), v1 = __half2float(vb[static_cast<size_t>(t + 1) * KW + d]);
      const float v2 = __half2float(vb[static_cast<size_t>(t + 2) * KW + d]), v3 = __half2float(vb[static_cast<size_t>(t + 3) * KW + d]);
      o = __fadd_rn(o, __fmul_rn(sc[t], v0));
      o = __fadd_rn(o, __fmul_rn(sc[t + 1], v1));
      o = __fadd_rn(o, __fmul_rn(sc[t + 2], v2));
      o = __fadd_rn(o, __fmul_rn(sc[t + 3], v3));
    }
    for (; t < n; ++t) o = __fadd_rn(o, __fmul_rn(sc[t], __half2float(vb[static_cast<size_t>(t) * KW + d])));
    a.att[static_cast<size_t>(b) * nq + h * hd + d] = o;
  }
}

// The same attention with one CTA per (key/value head, token) for all of the group's query heads: the keys and values pass
// through shared memory GA_BLK positions at a time (rows padded by 16 bytes, so the lanes of a warp, consecutive
// positions, read different banks), read once for the whole group. Scores: one thread per (head, position), the eight
// running sums of dotf_h; the maximum per head (a warp per head), e_t, the float sum in position order (a thread per head),
// p_t = e_t / sum; values: thread (head, d) chains in position order, a thread taking the same d of several heads so each
// staged value is read once for them. Shared memory: the group's queries [GRP][hd], the scores [GRP][pos + 1], the stage.
constexpr int GA_THREADS = 256, GA_BLK = 64;

__host__ __device__ inline size_t ga_smem(int grp, int hd, int n) {
  return static_cast<size_t>(grp) * hd * 4 + static_cast<size_t>(GA_BLK) * (hd + 8) * 2 + static_cast<size_t>(grp) * ((n + 3) & ~3) * 4 + 64;
}

__global__ void __launch_bounds__(GA_THREADS) attn_group_kernel(const PfAttnArgs a) {
  extern __shared__ __align__(16) uint8_t ga_sm[];
  __shared__ float s_mx[FWD_MAX_GROUP], s_sum[FWD_MAX_GROUP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = blockIdx.x, b = blockIdx.y, hd = a.hd, nq = a.n_head * hd, KW = a.n_kvw, GRP = a.n_head / a.n_kv;
  const int pos = a.pos0 + b, n = pos + 1, ns = (n + 3) & ~3, KS = hd + 8;
  float *qf = reinterpret_cast<float *>(ga_sm);                             // [GRP][hd]
  __half *kv = reinterpret_cast<__half *>(qf + GRP * hd);                   // [GA_BLK][hd + 8]
  float *sc = reinterpret_cast<float *>(kv + GA_BLK * KS);                  // [GRP][ns]
  for (int i = tid; i < GRP * hd; i += GA_THREADS) qf[i] = a.Qr[static_cast<size_t>(b) * nq + g * GRP * hd + i];
  const __half *kb = a.kc + g * hd, *vb = a.vc + g * hd;
  auto stage = [&](const __half *base, int b0, int cnt) {
    __syncthreads();
    for (int i = tid; i < cnt * (hd / 8); i += GA_THREADS) {
      const int t = i / (hd / 8), q = i - t * (hd / 8);
      *reinterpret_cast<uint4 *>(kv + t * KS + 8 * q) = reinterpret_cast<const uint4 *>(base + static_cast<size_t>(b0 + t) * KW)[q];
    }
    __syncthreads();
  };
  for (int b0 = 0; b0 < n; b0 += GA_BLK) {   // scores, the reference's dotf_h (c/src/forward.c:492-510)
    const int cnt = min(GA_BLK, n - b0);
    stage(kb, b0, cnt);
    for (int p = tid; p < GRP * GA_BLK; p += GA_THREADS) {
      const int j = p / GA_BLK, t = p - j * GA_BLK;
      if (t < cnt) {
        const __half *kr = kv + t * KS;
        const float *q = qf + j * hd;
        float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < hd; i += 8) {
          const uint4 kk = *reinterpret_cast<const uint4 *>(kr + i);
          const __half2 *k2 = reinterpret_cast<const __half2 *>(&kk);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 f = __half22float2(k2[u]);
            s8[2 * u] = __fadd_rn(s8[2 * u], __fmul_rn(q[i + 2 * u], f.x));
            s8[2 * u + 1] = __fadd_rn(s8[2 * u + 1], __fmul_rn(q[i + 2 * u + 1], f.y));
          }
        }
        const float d = __fadd_rn(__fadd_rn(__fadd_rn(s8[0], s8[1]), __fadd_rn(s8[2], s8[3])),
                                  __fadd_rn(__fadd_rn(s8[4], s8[5]), __fadd_rn(s8[6], s8[7])));
        sc[j * ns + b0 + t] = __fmul_rn(d, a.attn_scale);
      }
    }
  }
  __syncthreads();
  for (int j = warp; j < GRP; j += GA_THREADS / 32) {   // each head's maximum
    float mx = -INFINITY;
    for (int t = lane; t < n; t += 32) mx = fmaxf(mx, sc[j * ns + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0) s_mx[j] = mx;
  }
  __syncthreads();
  for (int i = tid; i < GRP * n; i += GA_THREADS) {
    const int j = i / n, t = i - j * n;
    sc[j * ns + t] = expf_cr(__fsub_rn(sc[j * ns + t], s_mx[j]));
  }
  __syncthreads();
  if (tid < GRP) {   // the float sum in position order (c/src/forward.c:602-603)
    float sum = 0.f;
    for (int t = 0; t < n; ++t) sum = __fadd_rn(sum, sc[tid * ns + t]);
    s_sum[tid] = sum;
  }
  __syncthreads();
  for (int i = tid; i < GRP * n; i += GA_THREADS) {
    const int j = i / n, t = i - j * n;
    sc[j * ns + t] = __fdiv_rn(sc[j * ns + t], s_sum[j]);
  }
  // values (axpy_h, c/src/forward.c:512-521): thread d of the head dimension takes heads j = jr, jr + JS, ...
  const int pairs = GRP * hd, JS = GA_THREADS / hd > 0 ? GA_THREADS / hd : 1;
  const int d = tid % hd, jr = tid / hd;
  constexpr int MAXJ = FWD_MAX_GROUP;
  float o[MAXJ];
#pragma unroll
  for (int k = 0; k < MAXJ; ++k) o[k] = 0.f;
  for (int b0 = 0; b0 < n; b0 += GA_BLK) {
    const int cnt = min(GA_BLK, n - b0);
    stage(vb, b0, cnt);
    if (tid < pairs && jr < JS) {
      for (int t = 0; t < cnt; ++t) {
        const float v = __half2float(kv[t * KS + d]);
#pragma unroll
        for (int k = 0; k < MAXJ; ++k) {
          const int j = jr + k * JS;
          if (j < GRP) o[k] = __fadd_rn(o[k], __fmul_rn(sc[j * ns + b0 + t], v));
        }
      }
    }
  }
  if (tid < pairs && jr < JS) {
#pragma unroll
    for (int k = 0; k < MAXJ; ++k) {
      const int j = jr + k * JS;
      if (j < GRP) a.att[static_cast<size_t>(b) * nq + (g * GRP + j) * hd + d] = o[k];
    }
  }
}

// Dense products of a batch: out [nb][rows] (= or += scale *) w [rows][cols] (Q4_K / Q6_K) times plain Q8_K activations.
// A CTA stages MT_ROWS rows (one bulk copy) and MT_TOK tokens' activations (swizzled Q8_K, each token's row padded by 16
// bytes so the lanes of a warp, one token each, read different banks); a warp takes a row at a time and every lane forms
// that row's dot product with its own token: the block terms of the reference (exact integer sums per 256-block) added in
// block order. The weights are read once per CTA (a broadcast to the warp's lanes).
constexpr int MT_ROWS = 32, MT_TOK = 32, MT_THREADS = 256;

struct MtLayout {
  uint32_t w, act, bs, dd, total, act_stride, bs_stride, dd_stride;
};
__host__ __device__ inline MtLayout mt_layout(uint32_t rb, int cols) {
  MtLayout L{};
  const uint32_t nblk = static_cast<uint32_t>(cols) / 256;
  L.w = 16;
  L.act = (L.w + MT_ROWS * rb + 32 + 15) & ~15u;
  L.act_stride = static_cast<uint32_t>(cols) + 16;
  L.bs = L.act + MT_TOK * L.act_stride;
  L.bs_stride = static_cast<uint32_t>(cols) / 16 + 2;   // int16 units: an odd number of words per token
  L.dd = (L.bs + MT_TOK * L.bs_stride * 2 + 15) & ~15u;
  L.dd_stride = nblk + 1;                               // floats: an odd number of words per token when nblk is even
  L.total = L.dd + MT_TOK * L.dd_stride * 4;
  return L;
}

__global__ void __launch_bounds__(MT_THREADS) mvt_kernel(const uint8_t *w, uint32_t type, uint32_t rb, int rows, int cols, int nb,
                                                         const int8_t *qs, const float *dd, const int16_t *bs, float *out,
                                                         int accum, float scale, int *err) {
  extern __shared__ __align__(128) uint8_t mt_sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * MT_ROWS, R = min(MT_ROWS, rows - r0);
  const int t0 = blockIdx.y * MT_TOK, nt = min(MT_TOK, nb - t0);
  const int nblk = cols / 256;
  const MtLayout L = mt_layout(rb, cols);
  uint64_t *bar = reinterpret_cast<uint64_t *>(mt_sm);
  const uint8_t *src = w + static_cast<size_t>(r0) * rb;
  const uint32_t lo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src) & 15u);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    const uint32_t n16 = (lo + static_cast<uint32_t>(R) * rb + 15u) & ~15u;
    mbar_arrive_expect_tx(bar, n16);
    bulk_copy_g2s(mt_sm + L.w, src - lo, n16, bar);
  }
  // this chunk's activations: values swizzled per 256-block (q8k_chunk_off), group sums and scales, rows padded
  const int chunks = cols / 16;
  for (int i = tid; i < nt * chunks; i += MT_THREADS) {
    const int t = i / chunks, c = i - t * chunks;
    const int4 v = *reinterpret_cast<const int4 *>(qs + static_cast<size_t>(t0 + t) * cols + 16 * c);
    *reinterpret_cast<int4 *>(mt_sm + L.act + t * L.act_stride + q8k_chunk_off(c >> 4, c & 15, true)) = v;
  }
  int16_t *sbs = reinterpret_cast<int16_t *>(mt_sm + L.bs);
  for (int i = tid; i < nt * chunks; i += MT_THREADS) {
    const int t = i / chunks, g = i - t * chunks;
    sbs[t * L.bs_stride + g] = bs[static_cast<size_t>(t0 + t) * chunks + g];
  }
  float *sdd = reinterpret_cast<float *>(mt_sm + L.dd);
  for (int i = tid; i < nt * nblk; i += MT_THREADS) {
    const int t = i / nblk, b = i - t * nblk;
    sdd[t * L.dd_stride + b] = dd[static_cast<size_t>(t0 + t) * nblk + b];
  }
  __syncthreads();
  if (!mbar_wait_bounded(bar, 0)) { set_error(err, ERR_WAIT_COPY); return; }
  if (lane >= nt) return;
  const SmemAct act{reinterpret_cast<const int8_t *>(mt_sm + L.act + lane * L.act_stride), sbs + lane * L.bs_stride, sdd + lane * L.dd_stride};
  const uint8_t *wrows = mt_sm + L.w + lo;
  for (int r = warp; r < R; r += MT_THREADS / 32) {
    const uint8_t *row = wrows + static_cast<size_t>(r) * rb;
    float sum = 0.f;
    for (int b = 0; b < nblk; ++b) sum = __fadd_rn(sum, kq_block_s<false>(type, row, b, act, b));
    float *o = out + static_cast<size_t>(t0 + lane) * rows + r0 + r;
    *o = accum ? __fadd_rn(*o, __fmul_rn(scale, sum)) : sum;
  }
}

__global__ void counts_kernel(int *co, int nb) {
  co[0] = nb;
  co[1] = 0;
  co[2] = nb;
}

__global__ void resid_add_kernel(float *x, const float *v, size_t n, float scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] = __fadd_rn(x[i], __fmul_rn(scale, v[i]));
}

}  // namespace

int pf_mv_tc(const FwdMat &m, int rows, int cols, int nb, const int8_t *qs, const float *dd, const int16_t *bs, float *out, int accum,
             float scale, const PfTc &tc, int *err, cudaStream_t st) {
  // the grouped kernel gives a dense matrix one CTA per (256-row tile, 64-token chunk): below 256 tokens too few to beat
  // the CUDA-core kernel's CTA per (32 rows, 32 tokens)
  if (m.type != T_Q4_K || nb < 256 || !tc_type_supported(T_Q4_K, m.p, rows, cols))
    return pf_mv(m, rows, cols, nb, qs, dd, bs, out, accum, scale, err, st);
  counts_kernel<<<1, 1, 0, st>>>(tc.co, nb);
  float *dst = accum ? tc.tmp : out;
  const int rc = launch_tc_dense(m.p, m.rb, rows, cols, nb, qs, dd, tc.co, tc.ph, tc.pl, tc.rs, dst, err, st);
  if (rc) return rc;
  if (accum) {
    const size_t n = static_cast<size_t>(nb) * rows;
    resid_add_kernel<<<static_cast<int>(std::min<size_t>((n + 255) / 256, 1184)), 256, 0, st>>>(out, tc.tmp, n, scale);
  }
  return static_cast<int>(cudaGetLastError());
}

int pf_mv(const FwdMat &m, int rows, int cols, int nb, const int8_t *qs, const float *dd, const int16_t *bs, float *out, int accum,
          float scale, int *err, cudaStream_t st) {
  if (nb < 8 || (m.type != T_Q4_K && m.type != T_Q6_K))
    return launch_mv_dev(m.p, m.type, rows, cols, nb, qs, dd, bs, out, accum, scale, err, st);
  const MtLayout L = mt_layout(m.rb, cols);
  if (L.total > 227 * 1024) return launch_mv_dev(m.p, m.type, rows, cols, nb, qs, dd, bs, out, accum, scale, err, st);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(mvt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr[dev] = true;
  }
  const dim3 grid((rows + MT_ROWS - 1) / MT_ROWS, (nb + MT_TOK - 1) / MT_TOK);
  mvt_kernel<<<grid, MT_THREADS, L.total, st>>>(m.p, m.type, m.rb, rows, cols, nb, qs, dd, bs, out, accum, scale, err);
  return static_cast<int>(cudaGetLastError());
}

cudaError_t pf_embed(const FwdMat &emb, const int *tok, int nb, int E, float embed_scale, float *X, cudaStream_t st) {
  embed_kernel<<<nb, PT, 0, st>>>(emb, tok, E, embed_scale, X);
  return cudaGetLastError();
}

cudaError_t pf_norm_q8k(const float *X, int row0, int nb, int E, const float *w, float eps, int8_t *qs, float *dd, int16_t *bs,
                        cudaStream_t st) {
  if (E > 4096 || E % 256) return cudaErrorInvalidValue;
  norm_q8k_kernel<<<nb, PT, 0, st>>>(X, row0, E, w, eps, qs, dd, bs);
  return cudaGetLastError();
}

cudaError_t pf_q8k(const float *src, int nb, int cols, int8_t *qs, float *dd, int16_t *bs, cudaStream_t st) {
  if (cols % 256) return cudaErrorInvalidValue;
  q8k_kernel<<<nb, PT, 0, st>>>(src, cols, qs, dd, bs);
  return cudaGetLastError();
}

cudaError_t pf_qk(const PfQkArgs &a, cudaStream_t st) {
  switch (a.hd) {
    case 64: qk_kernel<2><<<a.nb, PT, 0, st>>>(a); break;
    case 128: qk_kernel<4><<<a.nb, PT, 0, st>>>(a); break;
    case 256: qk_kernel<8><<<a.nb, PT, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t pf_attn(const PfAttnArgs &a, cudaStream_t st) {
  const int n = a.pos0 + a.nb;
  if (n > PF_MAX_CTX || a.hd % 8) return cudaErrorInvalidValue;
  const int grp = a.n_head / a.n_kv;
  const size_t gsm = ga_smem(grp, a.hd, n);
  if (grp <= FWD_MAX_GROUP && a.hd <= GA_THREADS && GA_THREADS % a.hd == 0 && gsm <= 200 * 1024) {   // the group kernel
    static bool gattr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !gattr[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(attn_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) return e;
      gattr[dev] = true;
    }
    attn_group_kernel<<<dim3(a.n_kv, a.nb), GA_THREADS, gsm, st>>>(a);
    return cudaGetLastError();
  }
  const size_t smem = (static_cast<size_t>(a.hd) + n) * 4;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (PF_MAX_CTX + 256) * 4);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  attn_kernel<<<dim3(a.n_head, a.nb), AT, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace clb
