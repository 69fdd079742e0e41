// The batched MoE block (T > 1 tokens): the reference's c/src/forward.c:1132-1210.
//
//   norm_kernel      per token: rmsnorm (double sum of squares), xn, Q8_K of xn
//   router_kernel    per (2 tokens, 32 experts), up to 512 tokens; router_chunked_kernel per (32 tokens, 32 experts)
//                    beyond: the reference's dotf logits, each router row read once for the CTA's tokens
//   topk_kernel      per token: softmax (double sum), top-k by repeated arg-max with ties to the lower id, renormalisation
//   dispatch_kernel  counting sort of the T*K (token, expert) slots by expert; each expert's tokens in ascending token order
//                    (the reference's who[] list, c/src/forward.c:1189-1190), plus each expert's first appearance and the
//                    experts in that order (the reference's todo[], c/src/forward.c:1163)
//   gateup_kernel    per (expert, 16 rows): gate and up row dots for every token of that expert (weights read once, staged
//                    in shared memory by a bulk copy), SwiGLU -> hg by dispatch position
//   hq_kernel        Q8_K of each hg row (K-quant down weights)
//   down_kernel      per (expert, 16 rows): down row dots for every token of that expert -> hd by dispatch position
//   combine_kernel   per (token, 512 columns): moe = sum over its experts in order of first appearance of wt*hd (the reference's todo
//                    order, c/src/forward.c:1163-1164), x += resid_scale * moe
#include <cstdio>
#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"
#include "rowdot.cuh"

namespace clb {

constexpr int BT = 256;          // threads of the batched kernels
constexpr int BNW = BT / 32;
constexpr int ROUTE_EXPERTS = BT / 8;
constexpr int ROWS_PER_CTA = 16; // weight rows per CTA in the expert kernels

// Per token: rmsnorm (double sum of squares, c/src/forward.c:412-417), xn to global memory (and its fp16 hi/lo planes for
// Q8_0 tensor-core experts), the Q8_K blocks of xn.
__global__ void __launch_bounds__(BT) norm_kernel(const BatchArgs a) {
  __shared__ double red[BNW];
  __shared__ __align__(16) float xs[4096];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, E = a.E;
  const float4 *x4 = reinterpret_cast<const float4 *>(a.x_in + static_cast<size_t>(t) * E);
  float *xn = a.xn + static_cast<size_t>(t) * E;
  double ss = 0.0;
  {   // the row (E <= 4096: at most four float4 a thread), all loads in flight, into shared memory
    float4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = u * BT + tid;
      r[u] = v < E / 4 ? x4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = u * BT + tid;
      if (v < E / 4) {
        reinterpret_cast<float4 *>(xs)[v] = r[u];
        ss += static_cast<double>(r[u].x) * r[u].x + static_cast<double>(r[u].y) * r[u].y +
              static_cast<double>(r[u].z) * r[u].z + static_cast<double>(r[u].w) * r[u].w;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  double tot = 0.0;
  for (int w = 0; w < BNW; ++w) tot += red[w];
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / static_cast<double>(E)), a.eps)));
  for (int i = tid; i < E; i += BT) {
    const float v = __fmul_rn(__fmul_rn(xs[i], scale), a.norm[i]);
    xs[i] = v;
    xn[i] = v;
    if (a.xh) {   // fp16 hi/lo planes of xn for the Q8_0 tensor-core products: xn = hi + lo to about 2^-22
      const __half h = __float2half_rn(v);
      a.xh[static_cast<size_t>(t) * E + i] = h;
      a.xl[static_cast<size_t>(t) * E + i] = __float2half_rn(__fsub_rn(v, __half2float(h)));
    }
  }
  __syncthreads();
  q8k_quantize_block(xs, E, a.xq_qs + static_cast<size_t>(t) * E, a.xq_d + static_cast<size_t>(t) * (E / 256),
                     a.xq_bs + static_cast<size_t>(t) * (E / 16), warp, BNW, lane);
}

// Router logits of ROUTER_TOKENS tokens x 32 experts per CTA, the reference's dotf (c/src/forward.c:574-581): eight lanes per
// expert, lane l summing w[i] * x[i] for i = l, l + 8, ... in element order, then ((0+1)+(2+3))+((4+5)+(6+7)). The tokens'
// xn rows sit in shared memory transposed by chain -- element i of token t at [t][i % 8][i / 8], rows padded by 4 floats so
// the eight chains fall in different banks -- so a lane reads its chain's next four elements with one 16-byte load, and a
// router row is read once for all the tokens.
// ROUTER_TOKENS: 2 tokens a CTA for batches up to 512 tokens (more CTAs); larger batches take router_chunked_kernel.
CLB_DEV int router_row(int E) { return E / 8 + 4; }   // floats per chain row
template <int ROUTER_TOKENS>
__global__ void __launch_bounds__(BT) router_kernel(const BatchArgs a) {
  extern __shared__ __align__(16) float xs[];   // [ROUTER_TOKENS][8][E/8 + 4]
  const int E = a.E, t0 = blockIdx.x * ROUTER_TOKENS, nt = min(ROUTER_TOKENS, a.T - t0), XR = router_row(E), XT = 8 * XR;
  const int tid = threadIdx.x, lane = tid & 31;
  {   // the tokens' rows: every load of a batch in flight before the transposing stores
    const int nvec = ROUTER_TOKENS * E / 4;
    const float4 *src = reinterpret_cast<const float4 *>(a.xn + static_cast<size_t>(t0) * E);
    for (int v0 = 0; v0 < nvec; v0 += 16 * BT) {
      float4 r[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int v = v0 + u * BT + tid;
        r[u] = (v < nvec && (4 * v) / E < nt) ? src[v] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int v = v0 + u * BT + tid;
        if (v < nvec) {
          const int t = (4 * v) / E, k = 4 * v - t * E;   // k is a multiple of 4: chains k%8 .. k%8+3, step k/8
          float *d = xs + t * XT + (k & 7) * XR + (k >> 3);
          d[0] = r[u].x;
          d[XR] = r[u].y;
          d[2 * XR] = r[u].z;
          d[3 * XR] = r[u].w;
        }
      }
    }
  }
  __syncthreads();
  const int grp = tid >> 3, l8 = tid & 7, e = blockIdx.y * ROUTE_EXPERTS + grp;
  float s[ROUTER_TOKENS];
#pragma unroll
  for (int t = 0; t < ROUTER_TOKENS; ++t) s[t] = 0.f;
  if (e < a.NE) {
    const float *w = a.router + static_cast<size_t>(e) * E;
    for (int k0 = 0; k0 < E / 8; k0 += 32) {   // chain steps k0 .. k0+31: 32 router loads in flight
      float wv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) wv[j] = __ldg(w + l8 + 8 * (k0 + j));
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
#pragma unroll
        for (int t = 0; t < ROUTER_TOKENS; ++t) {
          const float4 xv = *reinterpret_cast<const float4 *>(xs + t * XT + l8 * XR + k0 + 4 * j4);
          s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4], xv.x));
          s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4 + 1], xv.y));
          s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4 + 2], xv.z));
          s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4 + 3], xv.w));
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < ROUTER_TOKENS; ++t) {
    float p[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) p[l] = __shfl_sync(FULL, s[t], (lane & ~7) + l);
    if (t < nt && e < a.NE && l8 == 0)
      a.logits[static_cast<size_t>(t0 + t) * a.NE + e] =
          __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])), __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
  }
}

// Router logits for large batches: 32 tokens x 32 experts per CTA, so each router value is read once for 32 tokens. The
// tokens' xn rows pass through shared memory 512 elements at a time, transposed by chain as above; a lane's chain for
// each of the 32 tokens carries from one chunk to the next, so every chain adds its products in element order, the
// reference's dotf (c/src/forward.c:574-581), and the logits are the same bits as router_kernel's.
constexpr int RC_TOKENS = 32, RC_CHUNK = 512, RC_ROW = RC_CHUNK / 8 + 4;   // RC_ROW: floats per chain row of a chunk
constexpr int RC_SMEM = RC_TOKENS * 8 * RC_ROW * 4;
__global__ void __launch_bounds__(BT, 2) router_chunked_kernel(const BatchArgs a) {
  extern __shared__ __align__(16) float xs[];   // [RC_TOKENS][8][RC_ROW]
  const int E = a.E, t0 = blockIdx.x * RC_TOKENS, nt = min(RC_TOKENS, a.T - t0);
  const int tid = threadIdx.x, lane = tid & 31, grp = tid >> 3, l8 = tid & 7, e = blockIdx.y * ROUTE_EXPERTS + grp;
  const float *w = a.router + static_cast<size_t>(min(e, a.NE - 1)) * E;   // rows past NE read the last row, unused
  float s[RC_TOKENS];
#pragma unroll
  for (int t = 0; t < RC_TOKENS; ++t) s[t] = 0.f;
  for (int c0 = 0; c0 < E; c0 += RC_CHUNK) {
    const int ce = min(RC_CHUNK, E - c0), n4 = ce / 4;   // E is a multiple of 256: ce is 512 or 256
    __syncthreads();   // the previous chunk is consumed
    {   // every token's chunk: all loads in flight before the transposing stores
      constexpr int PER = RC_TOKENS * RC_CHUNK / 4 / BT;
      float4 r[PER];
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int v = u * BT + tid, t = v / n4, k4 = v - t * n4;
        r[u] = (t < nt) ? __ldcg(reinterpret_cast<const float4 *>(a.xn + static_cast<size_t>(t0 + t) * E + c0) + k4)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int v = u * BT + tid, t = v / n4, k = 4 * (v - t * n4);   // k a multiple of 4: chains k%8 .. k%8+3, step k/8
        if (t < RC_TOKENS) {
          float *d = xs + t * 8 * RC_ROW + (k & 7) * RC_ROW + (k >> 3);
          d[0] = r[u].x;
          d[RC_ROW] = r[u].y;
          d[2 * RC_ROW] = r[u].z;
          d[3 * RC_ROW] = r[u].w;
        }
      }
    }
    __syncthreads();
    if (e < a.NE) {
      for (int j0 = 0; j0 < ce / 8; j0 += 16) {   // chain steps j0 .. j0+15 of the chunk: 16 router loads in flight
        float wv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) wv[j] = __ldg(w + c0 + l8 + 8 * (j0 + j));
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
#pragma unroll
          for (int t = 0; t < RC_TOKENS; ++t) {
            const float4 xv = *reinterpret_cast<const float4 *>(xs + t * 8 * RC_ROW + l8 * RC_ROW + j0 + 4 * j4);
            s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4], xv.x));
            s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4 + 1], xv.y));
            s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4 + 2], xv.z));
            s[t] = __fadd_rn(s[t], __fmul_rn(wv[4 * j4 + 3], xv.w));
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < RC_TOKENS; ++t) {
    float p[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) p[l] = __shfl_sync(FULL, s[t], (lane & ~7) + l);
    if (t < nt && e < a.NE && l8 == 0)
      a.logits[static_cast<size_t>(t0 + t) * a.NE + e] =
          __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])), __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
  }
}

__global__ void __launch_bounds__(32) topk_kernel(const BatchArgs a) {
  const int t = blockIdx.x, lane = threadIdx.x, NE = a.NE, K = a.K;
  const float *lg = a.logits + static_cast<size_t>(t) * NE;
  float v[DECODE_MAX_NE / 32];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < DECODE_MAX_NE / 32; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < NE ? lg[e] : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  double sum = 0.0;
#pragma unroll
  for (int j = 0; j < DECODE_MAX_NE / 32; ++j)
    if (lane + 32 * j < NE) { v[j] = expf_cr(__fsub_rn(v[j], mx)); sum += static_cast<double>(v[j]); }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
  uint32_t used = 0;
#pragma unroll
  for (int j = 0; j < DECODE_MAX_NE / 32; ++j) {
    if (lane + 32 * j < NE) v[j] = __double2float_rn(__ddiv_rn(static_cast<double>(v[j]), sum));
    else used |= 1u << j;
  }
  __shared__ int s_sel[DECODE_MAX_K];
  __shared__ float s_wt[DECODE_MAX_K];
  for (int k = 0; k < K; ++k) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < DECODE_MAX_NE / 32; ++j)
      if (!((used >> j) & 1u) && (v[j] > bv || be == 0x7fffffff)) { bv = v[j]; be = lane + 32 * j; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, bv, o);
      const int oe = __shfl_xor_sync(FULL, be, o);
      if (oe != 0x7fffffff && (be == 0x7fffffff || ov > bv || (ov == bv && oe < be))) { bv = ov; be = oe; }
    }
    if ((be & 31) == lane) used |= 1u << (be >> 5);
    if (lane == 0) { s_sel[k] = be; s_wt[k] = bv; }
  }
  __syncwarp();
  if (lane == 0) {
    if (a.norm_topk) {
      float z = 0.f;
      for (int k = 0; k < K; ++k) z = __fadd_rn(z, s_wt[k]);
      if (z > 0.f) for (int k = 0; k < K; ++k) s_wt[k] = __fdiv_rn(s_wt[k], z);
    }
  }
  __syncwarp();
  for (int k = lane; k < K; k += 32) {
    const size_t i = static_cast<size_t>(t) * K + k;
    a.sel[i] = s_sel[k];
    a.wt[i] = s_wt[k];
    if (a.sel_out) a.sel_out[i] = s_sel[k];
    if (a.wt_out) a.wt_out[i] = s_wt[k];
  }
}

// One CTA. The (expert, token) pairs form a bit matrix (expert rows, token bits); an expert's tokens are its set bits in
// ascending order (the reference's who[] list, c/src/forward.c:1189-1190), so the dispatch position of slot (t, k) with
// expert e is offset[e] + the set bits of row e before bit t -- from a per-word prefix of population counts, in parallel
// over the slots.
__global__ void __launch_bounds__(1024) dispatch_kernel(const BatchArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int NE = a.NE, K = a.K, T = a.T, nw = (T + 31) / 32;
  uint32_t *bits = reinterpret_cast<uint32_t *>(sm);            // [NE][nw]
  int *wpre = reinterpret_cast<int *>(bits + NE * nw);          // [NE][nw] set bits of the row before word w
  int *cnt = wpre + NE * nw;                                    // [NE]
  int *off = cnt + NE;                                          // [NE + 1]
  int *first = off + NE + 1;                                    // [NE]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  for (int i = tid; i < NE * nw; i += blockDim.x) bits[i] = 0;
  for (int e = tid; e < NE; e += blockDim.x) first[e] = 0x7fffffff;
  __syncthreads();
  for (int s = tid; s < T * K; s += blockDim.x) {
    const int t = s / K, e = a.sel[s];
    if (e < 0 || e >= NE) {
      if (!(a.ep && e < 0)) set_error(a.err, ERR_BAD_EXPERT);   // -1: held by another GPU (expert-parallel)
      continue;
    }
    atomicOr(&bits[e * nw + t / 32], 1u << (t & 31));
    atomicMin(&first[e], s);
  }
  __syncthreads();
  for (int e = warp; e < NE; e += nwarps) {   // per expert: exclusive prefix of the words' population counts
    int base = 0;
    for (int w0 = 0; w0 < nw; w0 += 32) {
      const int w = w0 + lane;
      const int c = w < nw ? __popc(bits[e * nw + w]) : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) { const int v = __shfl_up_sync(FULL, incl, o); if (lane >= o) incl += v; }
      if (w < nw) wpre[e * nw + w] = base + incl - c;
      base += __shfl_sync(FULL, incl, 31);
    }
    if (lane == 0) cnt[e] = base;
  }
  __syncthreads();
  if (warp == 0) {   // exclusive prefix over the experts
    int base = 0;
    for (int e0 = 0; e0 < NE; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < NE ? cnt[e] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) { const int v = __shfl_up_sync(FULL, incl, o); if (lane >= o) incl += v; }
      if (e < NE) off[e] = base + incl - c;
      base += __shfl_sync(FULL, incl, 31);
    }
    if (lane == 0) off[NE] = base;
  }
  __syncthreads();
  for (int e = tid; e < NE; e += blockDim.x) {
    a.counts[e] = cnt[e];
    a.offsets[e] = off[e];
    a.first[e] = first[e];
    if (a.todo && cnt[e] > 0) {   // todo position = experts with tokens that appeared earlier (first slots are distinct)
      int r = 0;
      for (int f = 0; f < NE; ++f) r += cnt[f] > 0 && first[f] < first[e];
      a.todo[r] = e;
    }
  }
  if (tid == 0) a.offsets[NE] = off[NE];
  if (a.todo && warp == 0) {
    int n = 0;
    for (int e = lane; e < NE; e += 32) n += cnt[e] > 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(FULL, n, o);
    if (lane == 0) a.todo[NE] = n;
  }
  for (int s = tid; s < T * K; s += blockDim.x) {
    const int t = s / K, e = a.sel[s];
    if (e < 0 || e >= NE) continue;
    const int w = t / 32;
    const int pos = off[e] + wpre[e * nw + w] + __popc(bits[e * nw + w] & ((1u << (t & 31)) - 1u));
    a.pos_token[pos] = t;
    a.pos_wt[pos] = a.wt[s];
    a.slot_pos[s] = pos;
  }
}

// gate and up rows [r0, r0+R) of expert e for each of its tokens.
__global__ void __launch_bounds__(BT) gateup_kernel(const BatchArgs a) {
  const int e = blockIdx.x, n = a.counts[e];
  if (n == 0) return;
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, E = a.E, FF = a.FF;
  const int r0 = blockIdx.y * ROWS_PER_CTA, R = min(ROWS_PER_CTA, FF - r0);
  const uint32_t grb = a.grb;
  const uint32_t seg = (R * grb + 32 + 15) & ~15u;
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
  float *xf = reinterpret_cast<float *>(sm + 16);                          // [E] (Q8_0: the token's xn)
  float *res = xf + E;                                                     // [2 * ROWS_PER_CTA]
  uint8_t *wbuf = reinterpret_cast<uint8_t *>(res + 2 * ROWS_PER_CTA);
  const uint8_t *sg = a.gate + static_cast<size_t>(e) * a.gate_slab + static_cast<size_t>(r0) * grb;
  const uint8_t *su = a.up + static_cast<size_t>(e) * a.up_slab + static_cast<size_t>(r0) * grb;
  const uint32_t lg = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(sg) & 15u), lu = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(su) & 15u);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    const uint32_t ng = (lg + R * grb + 15u) & ~15u, nu = (lu + R * grb + 15u) & ~15u;
    mbar_arrive_expect_tx(bar, ng + nu);
    bulk_copy_g2s(wbuf, sg - lg, ng, bar);
    bulk_copy_g2s(wbuf + seg, su - lu, nu, bar);
  }
  __syncthreads();
  const uint8_t *g = wbuf + lg, *u = wbuf + seg + lu;
  const int p0 = a.offsets[e];
  if (p0 < 0 || n < 0 || p0 + n > a.T * a.K) { set_error(a.err, ERR_BAD_EXPERT); mbar_wait_bounded(bar, 0); return; }
  const bool q80 = a.gate_type == T_Q8_0;
  const int nb = q80 ? E / 32 : E / 256;
  const RowShape rs = row_shape(q80 ? nb : 4 * nb);
  const int sub = lane / rs.LG, lig = lane % rs.LG;
  if (!mbar_wait_bounded(bar, 0)) { set_error(a.err, ERR_WAIT_COPY); return; }
  for (int i = 0; i < n; ++i) {
    const int pos = p0 + i, t = a.pos_token[pos];
    if (t < 0 || t >= a.T) { set_error(a.err, ERR_BAD_EXPERT); return; }
    KQAct act;
    if (q80) {
      __syncthreads();
      for (int j = tid; j < E; j += BT) xf[j] = a.xn[static_cast<size_t>(t) * E + j];
      __syncthreads();
    } else {
      load_kq_act(a.gate_type, a.xq_qs + static_cast<size_t>(t) * E, a.xq_d + static_cast<size_t>(t) * (E / 256),
                  a.xq_bs + static_cast<size_t>(t) * (E / 16), nb, rs, lig, act);
    }
    for (int base = warp * rs.RPW; base < 2 * R; base += BNW * rs.RPW) {
      const int task = base + sub;
      const bool active = sub < rs.RPW && task < 2 * R;
      const int r = task < R ? task : task - R;
      const uint8_t *row = (task < R ? g : u) + static_cast<size_t>(active ? r : 0) * grb;
      const float v = q80 ? q80_row(row, nb, rs, lig, sub * rs.LG, xf, active) : kq_row(a.gate_type, row, nb, rs, lig, sub * rs.LG, act, active);
      if (active && lig == 0) res[task] = v;
    }
    __syncthreads();
    for (int r = tid; r < R; r += BT) a.hg[static_cast<size_t>(pos) * FF + r0 + r] = silu_mul(res[r], res[R + r]);
    __syncthreads();
  }
}

__global__ void hq_kernel(const BatchArgs a, int npos) {
  const int pos = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, FF = a.FF;
  if (pos >= npos || pos >= a.offsets[a.NE]) return;   // only dispatched slots hold an hg row
  q8k_quantize_block(a.hg + static_cast<size_t>(pos) * FF, FF, a.hq_qs + static_cast<size_t>(pos) * FF,
                     a.hq_d + static_cast<size_t>(pos) * (FF / 256), a.hq_bs + static_cast<size_t>(pos) * (FF / 16), warp,
                     blockDim.x >> 5, lane);
}

// down rows [r0, r0+R) of expert e for each of its tokens.
__global__ void __launch_bounds__(BT) down_kernel(const BatchArgs a) {
  const int e = blockIdx.x, n = a.counts[e];
  if (n == 0) return;
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, E = a.E, FF = a.FF;
  const int r0 = blockIdx.y * ROWS_PER_CTA, R = min(ROWS_PER_CTA, E - r0);
  const uint32_t drb = a.drb;
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
  float *xf = reinterpret_cast<float *>(sm + 16);   // [FF] (Q8_0: the token's hg)
  uint8_t *wbuf = reinterpret_cast<uint8_t *>(xf + FF);
  const uint8_t *src = a.down + static_cast<size_t>(e) * a.down_slab + static_cast<size_t>(r0) * drb;
  const uint32_t lo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src) & 15u);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    const uint32_t n16 = (lo + R * drb + 15u) & ~15u;
    mbar_arrive_expect_tx(bar, n16);
    bulk_copy_g2s(wbuf, src - lo, n16, bar);
  }
  __syncthreads();
  const uint8_t *rows = wbuf + lo;
  const bool q80 = a.down_type == T_Q8_0;
  const int nb = q80 ? FF / 32 : FF / 256;
  const RowShape rs = row_shape(q80 ? nb : 4 * nb);
  const int sub = lane / rs.LG, lig = lane % rs.LG;
  if (!mbar_wait_bounded(bar, 0)) { set_error(a.err, ERR_WAIT_COPY); return; }
  const int p0 = a.offsets[e];
  if (p0 < 0 || n < 0 || p0 + n > a.T * a.K) { set_error(a.err, ERR_BAD_EXPERT); return; }
  for (int i = 0; i < n; ++i) {
    const int pos = p0 + i;
    KQAct act;
    if (q80) {
      __syncthreads();
      for (int j = tid; j < FF; j += BT) xf[j] = a.hg[static_cast<size_t>(pos) * FF + j];
      __syncthreads();
    } else {
      load_kq_act(a.down_type, a.hq_qs + static_cast<size_t>(pos) * FF, a.hq_d + static_cast<size_t>(pos) * (FF / 256),
                  a.hq_bs + static_cast<size_t>(pos) * (FF / 16), nb, rs, lig, act);
    }
    for (int base = warp * rs.RPW; base < R; base += BNW * rs.RPW) {
      const int r = base + sub;
      const bool active = sub < rs.RPW && r < R;
      const uint8_t *row = rows + static_cast<size_t>(active ? r : 0) * drb;
      const float v = q80 ? q80_row(row, nb, rs, lig, sub * rs.LG, xf, active) : kq_row(a.down_type, row, nb, rs, lig, sub * rs.LG, act, active);
      if (active && lig == 0) a.hd[static_cast<size_t>(pos) * E + r0 + r] = v;
    }
  }
}

// K-quant down rows of the integer path for experts with several tokens: two threads per row (DR rows of expert e staged by
// one bulk copy; each thread takes half of every block's groups), every token of the expert against the row in passes of
// 8, 4, 2 or 1 tokens (their Q8_K hg rows in shared memory, read by all threads at once), so each weight word is unpacked
// once per pass. The two halves' exact integer sums meet by a shuffle; then the reference's block term per token (Q6_K:
// d * d_a * sum_g sc_g (dot_g - 32 bsum_g); Q4_K: d_a * (d * sum_j sc_j dot_j - dmin * sum_j mn_j bsum_j)), added in
// block order.
constexpr int DR = 128, DRT = 2 * DR, DCH = 32;   // rows, threads, tokens staged at once

__host__ __device__ inline size_t down_rows_act_bytes(int FF) { return static_cast<size_t>(DCH) * (FF + FF / 256 * 4 + FF / 16 * 2); }

// One pass of NT tokens (staged rows t0 .. t0 + NT - 1) over the row: writes their outputs to hd (thread half 0).
template <uint32_t DT, int NT>
CLB_DEV void down_pass(const BatchArgs &a, const uint8_t *row, int half, const int8_t *aq, const int16_t *ab, const float *ad,
                       int t0, size_t pos0, int col, bool store) {
  const int FF = a.FF, nbd = FF / 256, nbs = FF / 16;
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  for (int blk = 0; blk < nbd; ++blk) {
    int si[NT], mi[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) si[t] = mi[t] = 0;
    const int8_t *xq = aq + static_cast<size_t>(t0) * FF + 256 * blk;
    const int16_t *xb = ab + t0 * nbs + 16 * blk;
    if (DT == T_Q6_K) {
      const uint8_t *bp = row + 210 * blk;
      const int8_t *sc = reinterpret_cast<const int8_t *>(bp + 192);
#pragma unroll 2
      for (int g = 8 * half; g < 8 * half + 8; ++g) {   // 16-groups: half h, part (which 32 of the half), which 16
        const int h = g >> 3, part = (g & 7) >> 1, l0 = 16 * (g & 1);
        const uint8_t *ql = bp + 64 * h + l0 + 32 * (part & 1), *qh = bp + 128 + 32 * h + l0;
        uint32_t v[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const uint32_t L = lds_u32_unaligned(ql + 4 * w), H = lds_u32_unaligned(qh + 4 * w);
          v[w] = ((part >= 2 ? (L >> 4) : L) & 0x0f0f0f0fu) | (((H >> (2 * part)) & 0x03030303u) << 4);
        }
        const int s = sc[g];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int4 x = reinterpret_cast<const int4 *>(xq + t * FF)[g];
          int d = __dp4a(static_cast<int>(v[0]), x.x, 0);
          d = __dp4a(static_cast<int>(v[1]), x.y, d);
          d = __dp4a(static_cast<int>(v[2]), x.z, d);
          d = __dp4a(static_cast<int>(v[3]), x.w, d);
          si[t] += s * (d - 32 * xb[t * nbs + g]);
        }
      }
    } else {   // Q4_K: 64-value groups g4 (low nibbles sub-block 2 g4, high nibbles 2 g4 + 1), two per thread
      const uint8_t *bp = row + 144 * blk;
#pragma unroll 1
      for (int g4 = 2 * half; g4 < 2 * half + 2; ++g4) {
        int sc0, mn0, sc1, mn1;
        q4k_scale_min(bp + 4, 2 * g4, sc0, mn0);
        q4k_scale_min(bp + 4, 2 * g4 + 1, sc1, mn1);
        uint32_t wq[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) wq[w] = lds_u32_unaligned(bp + 16 + 32 * g4 + 4 * w);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int4 *xa = reinterpret_cast<const int4 *>(xq + t * FF + 64 * g4);
          const int4 x0 = xa[0], x1 = xa[1], x2 = xa[2], x3 = xa[3];
          const int xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w}, xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
          int l = 0, hh = 0;
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            l = __dp4a(static_cast<int>(wq[w] & 0x0f0f0f0fu), xl[w], l);
            hh = __dp4a(static_cast<int>((wq[w] >> 4) & 0x0f0f0f0fu), xh[w], hh);
          }
          const int16_t *b16 = xb + t * nbs + 4 * g4;
          si[t] += sc0 * l + sc1 * hh;
          mi[t] += mn0 * (b16[0] + b16[1]) + mn1 * (b16[2] + b16[3]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {   // the row's two halves: exact integer sums, any order
      si[t] += __shfl_xor_sync(0xffffffffu, si[t], 1);
      if (DT == T_Q4_K) mi[t] += __shfl_xor_sync(0xffffffffu, mi[t], 1);
    }
    if (DT == T_Q6_K) {
      const float dw = f16_bits_to_f32(lds_u16(row + 210 * blk + 208));
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(dw, ad[(t0 + t) * nbd + blk]), static_cast<float>(si[t])));
    } else {
      const uint8_t *bp = row + 144 * blk;
      const float dw = f16_bits_to_f32(lds_u16(bp)), dmin = f16_bits_to_f32(lds_u16(bp + 2));
#pragma unroll
      for (int t = 0; t < NT; ++t)
        acc[t] = __fadd_rn(acc[t], __fmul_rn(ad[(t0 + t) * nbd + blk], __fsub_rn(__fmul_rn(dw, static_cast<float>(si[t])),
                                                                               __fmul_rn(dmin, static_cast<float>(mi[t])))));
    }
  }
  if (store) {
#pragma unroll
    for (int t = 0; t < NT; ++t) a.hd[(pos0 + t) * a.E + col] = acc[t];
  }
}

template <uint32_t DT>
__global__ void __launch_bounds__(DRT) down_rows_kernel(const BatchArgs a) {
  const int e = blockIdx.x, n = a.counts[e];
  if (n == 0) return;
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, half = tid & 1, rr = tid >> 1, E = a.E, FF = a.FF, nbd = FF / 256;
  const int r0 = blockIdx.y * DR, R = min(DR, E - r0);
  const uint32_t drb = a.drb;
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
  int8_t *aq = reinterpret_cast<int8_t *>(sm + 16);                               // [DCH][FF]
  float *ad = reinterpret_cast<float *>(aq + DCH * FF);                           // [DCH][nbd]
  int16_t *ab = reinterpret_cast<int16_t *>(ad + DCH * nbd);                      // [DCH][FF / 16]
  uint8_t *wbuf = sm + ((16 + down_rows_act_bytes(FF) + 15) & ~size_t(15));
  const uint8_t *src = a.down + static_cast<size_t>(e) * a.down_slab + static_cast<size_t>(r0) * drb;
  const uint32_t lo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src) & 15u);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    const uint32_t n16 = (lo + R * drb + 15u) & ~15u;
    mbar_arrive_expect_tx(bar, n16);
    bulk_copy_g2s(wbuf, src - lo, n16, bar);
  }
  __syncthreads();
  const int p0 = a.offsets[e];
  const bool bad = p0 < 0 || n < 0 || p0 + n > a.T * a.K;
  if (bad && tid == 0) set_error(a.err, ERR_BAD_EXPERT);
  if (!mbar_wait_bounded(bar, 0)) { set_error(a.err, ERR_WAIT_COPY); return; }
  if (bad) return;
  const bool live = rr < R;
  const uint8_t *row = wbuf + lo + static_cast<size_t>(live ? rr : 0) * drb;
  for (int s0 = 0; s0 < n; s0 += DCH) {
    const int ns = min(DCH, n - s0);
    __syncthreads();   // the previous tokens' activations are consumed
    for (int i = tid; i < ns * (FF / 16); i += DRT) {
      const int t = i / (FF / 16), c = i - t * (FF / 16);
      reinterpret_cast<int4 *>(aq + t * FF)[c] = reinterpret_cast<const int4 *>(a.hq_qs + static_cast<size_t>(p0 + s0 + t) * FF)[c];
      ab[t * (FF / 16) + c] = a.hq_bs[static_cast<size_t>(p0 + s0 + t) * (FF / 16) + c];
    }
    for (int i = tid; i < ns * nbd; i += DRT) ad[i] = a.hq_d[static_cast<size_t>(p0 + s0) * nbd + i];
    __syncthreads();
    const bool store = live && half == 0;
    const size_t pos = static_cast<size_t>(p0 + s0);
    int t = 0;   // passes of 8, then 4, 2, 1 tokens: the same sequence in every thread (the shuffles)
    for (; t + 8 <= ns; t += 8) down_pass<DT, 8>(a, row, half, aq, ab, ad, t, pos + t, r0 + rr, store);
    if (t + 4 <= ns) { down_pass<DT, 4>(a, row, half, aq, ab, ad, t, pos + t, r0 + rr, store); t += 4; }
    if (t + 2 <= ns) { down_pass<DT, 2>(a, row, half, aq, ab, ad, t, pos + t, r0 + rr, store); t += 2; }
    if (t < ns) down_pass<DT, 1>(a, row, half, aq, ab, ad, t, pos + t, r0 + rr, store);
  }
}

// Per (token, 512 columns): the token's experts in order of first appearance, weighted, plus the residual.
__global__ void __launch_bounds__(BT) combine_kernel(const BatchArgs a) {
  const int t = blockIdx.x, K = a.K, E = a.E, i0 = blockIdx.y * 2 * BT, i1 = min(E, i0 + 2 * BT);
  __shared__ int s_pos[DECODE_MAX_K];
  __shared__ float s_w[DECODE_MAX_K];
  __shared__ int s_n;
  if (threadIdx.x == 0) {
    int order[DECODE_MAX_K], key[DECODE_MAX_K], n = 0;
    for (int k = 0; k < K; ++k) {   // insertion sort of the token's slots by their expert's first appearance
      const int e = a.sel[static_cast<size_t>(t) * K + k];
      if (e < 0 && a.ep) continue;  // held by another GPU
      const int kk = (e >= 0 && e < a.NE) ? a.first[e] : 0x7fffffff;
      int j = n;
      while (j > 0 && key[j - 1] > kk) { key[j] = key[j - 1]; order[j] = order[j - 1]; --j; }
      key[j] = kk; order[j] = k;
      ++n;
    }
    for (int j = 0; j < n; ++j) {
      s_pos[j] = a.slot_pos[static_cast<size_t>(t) * K + order[j]];
      s_w[j] = a.wt[static_cast<size_t>(t) * K + order[j]];
    }
    s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  if (a.ep && n == 0) return;   // a row with no expert here (an exchange's unused row): nothing reads its partial sum
  for (int j = 0; j < n; ++j)
    if (s_pos[j] < 0 || s_pos[j] >= a.T * K) { if (threadIdx.x == 0) set_error(a.err, ERR_BAD_EXPERT); return; }
  for (int i = i0 + threadIdx.x; i < i1; i += BT) {
    float m = 0.f;
    for (int j = 0; j < n; ++j) m = __fadd_rn(m, __fmul_rn(s_w[j], a.hd[static_cast<size_t>(s_pos[j]) * E + i]));
    const size_t xi = static_cast<size_t>(t) * E + i;
    a.x_out[xi] = a.ep ? m : __fadd_rn(a.x_in[xi], __fmul_rn(a.resid_scale, m));
  }
}

static size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

int launch_route(const BatchArgs &a, void *stream_) {
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {};
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(router_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RC_SMEM);
    cudaFuncSetAttribute(router_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 8 * (4096 / 8 + 4) * 4);
    attr[dev] = true;
  }
  norm_kernel<<<a.T, BT, 0, st>>>(a);
  const int eg = (a.NE + ROUTE_EXPERTS - 1) / ROUTE_EXPERTS;
  if (a.T > 512) router_chunked_kernel<<<dim3((a.T + RC_TOKENS - 1) / RC_TOKENS, eg), BT, RC_SMEM, st>>>(a);
  else router_kernel<2><<<dim3((a.T + 1) / 2, eg), BT, 2 * 8 * (a.E / 8 + 4) * 4, st>>>(a);
  topk_kernel<<<a.T, 32, 0, st>>>(a);
  return static_cast<int>(cudaGetLastError());
}

int launch_batched(const BatchArgs &a, void *stream_) {
  const int rc = launch_route(a, stream_);
  return rc ? rc : launch_experts(a, stream_);
}

int launch_dispatch(const BatchArgs &a, void *stream_) {
  const int nw = (a.T + 31) / 32;
  const size_t disp_smem = static_cast<size_t>(a.NE) * nw * 8 + (3 * a.NE + 1) * 4;
  if (disp_smem > 200 * 1024) return static_cast<int>(cudaErrorInvalidValue);   // tokens x experts beyond one CTA's bit matrix
  cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  dispatch_kernel<<<1, 1024, disp_smem, static_cast<cudaStream_t>(stream_)>>>(a);
  return static_cast<int>(cudaGetLastError());
}

int launch_experts(const BatchArgs &a, void *stream_) {
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int T = a.T, E = a.E, FF = a.FF, NE = a.NE, K = a.K;
  const int nw = (T + 31) / 32;
  const size_t disp_smem = static_cast<size_t>(NE) * nw * 8 + (3 * NE + 1) * 4;
  if (disp_smem > 200 * 1024) return static_cast<int>(cudaErrorInvalidValue);   // tokens x experts beyond one CTA's bit matrix
  dispatch_kernel<<<1, 1024, disp_smem, st>>>(a);
  const size_t gu_smem = 16 + E * 4 + 2 * ROWS_PER_CTA * 4 + 2 * align16(ROWS_PER_CTA * a.grb + 32) + 16;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attrs[64] = {};
  if (dev < 64 && !attrs[dev]) {   // per device: the attribute belongs to the current device's context
    cudaFuncSetAttribute(gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(down_rows_kernel<T_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(down_rows_kernel<T_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attrs[dev] = true;
  }
  if (a.tc_gu) {   // grouped GEMMs on the tensor cores
    const int rc = launch_tc(a, stream_, true);
    if (rc) return rc;
  } else {
    gateup_kernel<<<dim3(NE, (FF + ROWS_PER_CTA - 1) / ROWS_PER_CTA), BT, gu_smem, st>>>(a);
  }
  if (a.down_type != T_Q8_0) hq_kernel<<<T * K, 32 * (FF / 256), 0, st>>>(a, T * K);   // Q8_K of hg (K-quant down)
  if (a.tc_dn) {
    const int rc = launch_tc(a, stream_, false);
    if (rc) return rc;
  } else if (a.down_type == T_Q6_K || a.down_type == T_Q4_K) {
    const size_t dr_smem = align16(16 + down_rows_act_bytes(FF)) + align16(DR * a.drb + 32);
    if (dr_smem > 200 * 1024) return static_cast<int>(cudaErrorInvalidValue);
    const dim3 grid(NE, (E + DR - 1) / DR);
    if (a.down_type == T_Q6_K) down_rows_kernel<T_Q6_K><<<grid, DRT, dr_smem, st>>>(a);
    else down_rows_kernel<T_Q4_K><<<grid, DRT, dr_smem, st>>>(a);
  } else {
    const size_t dn_smem = 16 + FF * 4 + align16(ROWS_PER_CTA * a.drb + 32) + 16;
    down_kernel<<<dim3(NE, (E + ROWS_PER_CTA - 1) / ROWS_PER_CTA), BT, dn_smem, st>>>(a);
  }
  combine_kernel<<<dim3(T, (E + 2 * BT - 1) / (2 * BT)), BT, 0, st>>>(a);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace clb
