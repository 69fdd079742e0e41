// The one-token MoE block with each chosen expert owned by a group of CTAs: the reference's c/src/forward.c:949-1033 on
// one B200, laid out so that no step waits on the whole grid except the routing.
//
// Grid: K groups of ne = floor(SMs / K) CTAs (one per SM, 512 threads). CTA c < NE also scores expert c (c + G, ... when
// there are more experts than CTAs); CTAs that neither score nor work exit at once. Group k streams the expert at rank k:
// CTA i of it holds gate and up rows [FF*i/ne, FF*(i+1)/ne) and down rows [E*i/ne, E*(i+1)/ne) of that expert, so every
// byte of the chosen experts is read once, split evenly over the groups.
//
//   0  (before the programmatic-launch wait, overlapping the previous kernel's tail) mbarriers; the norm weights and the
//      router rows this CTA scores start streaming into shared memory;
//   1  x into shared memory, the double sum of squares, xn = rmsnorm(x) (c/src/forward.c:412-417);
//   2  the products router row x xn are laid out per strided chain; the last warp adds them in the reference's dotf order
//      (c/src/forward.c:574-581: eight strided float chains in element order, combined ((0+1)+(2+3))+((4+5)+(6+7))) and
//      publishes each logit as a self-tagged word (value and launch tag in one 64-bit store: no counter, no second round
//      trip); the other warps form the Q8_K blocks of xn;
//   3  every worker gathers the NE logit words and ranks the experts by logit (ties to the lower id), each warp a share of
//      them by warp reductions over the logits in registers. Softmax is monotone, so this is the reference's probability
//      order (c/src/forward.c:975-980) except where two different logits round to the same probability; the copies go out
//      on this order at once;
//   4  lanes of warp 0 issue the bulk copies of this CTA's rows of its group's expert: gate and up rows in row groups (one
//      mbarrier each, so compute follows the data in), then the down rows;
//   5  while they fly, the last warp alone forms the softmax (c/src/forward.c:954-958; the double sum in expert order, or
//      in any order where every term is a multiple of 2^-45 and the sum is exact), the probability order among the experts
//      that can reach the top k, and the renormalised weights (c/src/forward.c:984), and hands its verdict to the gate/up
//      warps through a named barrier. A group whose expert is not in the true top-k (a probability tie at rank k) waits
//      for its copies and fetches the right expert: the result is the reference's in every case;
//   6  gate/up rows (the other warps): a group of lanes per row, one lane per 256-block (exact integer sums, the
//      reference's float block term), the terms added in block order, SwiGLU (c/src/forward.c:1018); each hg value goes
//      out as a self-tagged word;
//   7  the group's FF hg words gathered, its Q8_K blocks formed once per CTA (c/src/quant.c:195-206), the down rows' block
//      terms (a warp's lanes share one activation block), hd = the terms in block order, wt * hd out as self-tagged words;
//   8  the combiner of row chunk i (CTA i of group i mod K) gathers the other groups' weighted rows of the chunk, adds the K
//      of them in rank order and writes x = x + resid_scale * moe (c/src/forward.c:1026-1032). The others exit.
// The combiner of chunk 0 (CTA 0) advances the launch generation, the tag of the next launch's words: by then every CTA
// that reads it has read it (each one's words were needed on the way).
#include "common.cuh"
#include "decode.cuh"
#include "rowdot.cuh"

namespace clb {

namespace {

constexpr int NW = GROUP_THREADS / 32;
constexpr int SW = NW - 1;                 // the scoring and softmax warp; warps 0..SW-1 take the gate/up rows
constexpr int NJ_MAX = GROUP_MAX_NE / 32;  // experts per lane in the warp-register ranking

// Shared-memory scalars.
struct GroupMisc {
  double red[NW];
  int flag[4];                   // [0] failed, [1] rounds of copies issued, [2] generation advanced, [3] expert to refetch + 1
  int tiny;                      // a softmax term below 2^-22: the double sum is taken in expert order
  int spec[DECODE_MAX_K + 1];    // experts by logit rank (rank K kept for the test hook)
  int top;                       // the expert with the largest logit
  int tru[DECODE_MAX_K];         // experts by probability rank (the reference's order)
  int slot[DECODE_MAX_K];        // probability rank -> the group that streams that expert
  float w[DECODE_MAX_K];         // renormalised weights by probability rank
  float mine;                    // this CTA's group's weight
};

CLB_DEV uint32_t fbits(float v) { return __float_as_uint(v); }

// Words i in [0, n) (at addr(i)) into dst(i) (floats), by `nt` threads from thread `t`: each thread polls its words (up to
// 8) together, so the round trips overlap. False when the limit ran out.
template <typename Addr, typename Dst>
CLB_DEV bool gather_words(Addr addr, Dst dst, int n, uint32_t tag, int t, int nt) {
  constexpr int MAXW = 8;
  uint32_t have = 0, want = 0;
#pragma unroll
  for (int q = 0; q < MAXW; ++q)
    if (t + q * nt < n) want |= 1u << q;
#pragma unroll 1
  for (uint32_t it = 0; it < SPIN_LIMIT && have != want; ++it) {
#pragma unroll
    for (int q = 0; q < MAXW; ++q) {
      const int i = t + q * nt;
      if (((want & ~have) >> q) & 1u) {
        const unsigned long long v = ld_word(addr(i));
        if (static_cast<uint32_t>(v >> 32) == tag) { *dst(i) = __uint_as_float(static_cast<uint32_t>(v)); have |= 1u << q; }
      }
    }
    if (it > 4096 && have != want) __nanosleep(64);
  }
  return have == want;
}
CLB_DEV void named_sync(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }
CLB_DEV void named_arrive(int n) { asm volatile("bar.arrive 1, %0;" ::"r"(n) : "memory"); }
CLB_DEV void fail(const GroupArgs &a, GroupMisc &m, int code) {
  set_error(a.err, code);
  m.flag[0] = 1;
  if (a.err_out) *reinterpret_cast<volatile int *>(a.err_out) = code;
}

// Ranks of the many-ties case (more than 32 experts can reach the top k, for example every logit equal): each candidate e
// by a warp count of the experts ahead of it. Out of line: it runs only in degenerate cases.
__device__ __noinline__ void rank_all_candidates(GroupMisc &m, const float *sp, int NE, int K, float pk, int lane) {
  for (int e = 0; e < NE; ++e) {
    const float pe = sp[e];
    if (!(pe >= pk)) continue;   // warp-uniform
    int rank = 0;
    for (int f0 = 0; f0 < NE; f0 += 32) {
      const int f = f0 + lane;
      const float pf = f < NE ? sp[f] : -1.f;
      rank += __popc(__ballot_sync(FULL, f < NE && (pf > pe || (pf == pe && f < e))));
    }
    if (lane == 0 && rank < K) m.tru[rank] = e;
  }
}

// Q8_K blocks of n floats (shared memory), out of line so its two uses share one copy of the code.
__device__ __noinline__ void q8k_blocks(const float *x, int n, int8_t *qs, float *dd, int16_t *bsums, int warp, int nwarps, int lane) {
  q8k_quantize_block(x, n, qs, dd, bsums, warp, nwarps, lane, true);
}

// The softmax warps (the warps without gate/up rows; the last of them finishes alone): probabilities, the reference's top-k
// order, the weights and which group streams which expert (c/src/forward.c:954-984). lg [NE] logits; kg this CTA's group;
// st = this thread's index among the nst softmax threads. The loops stay rolled: this code runs once a launch.
__device__ __noinline__ void softmax_verdict(const GroupArgs &a, GroupMisc &m, const float *lg, float *sev, float *sp, int kg,
                                             int st, int nst, bool cta0) {
  const int NE = a.NE, K = a.K, lane = st & 31;
  const float mx = lg[m.top];
  bool tiny = false;
#pragma unroll 1
  for (int e = st; e < NE; e += nst) {
    const float v = expf_cr(__fsub_rn(lg[e], mx));
    sev[e] = v;
    tiny |= !(v >= 0x1p-22f);
  }
  if (tiny) m.tiny = 1;
  asm volatile("bar.sync 2, %0;" ::"r"(nst) : "memory");
  // Every term a multiple of 2^-45 (each is a float >= 2^-22) and the sum below 2^8: every partial sum is exact in any
  // order, so a tree gives the reference's sequential double sum; otherwise it is added in expert order. Every softmax
  // warp forms the same sum.
  double sum = 0.0;
  if (!m.tiny) {
#pragma unroll 1
    for (int e = lane; e < NE; e += 32) sum += static_cast<double>(sev[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
  } else {
    if (lane == 0)
      for (int e = 0; e < NE; ++e) sum += static_cast<double>(sev[e]);
    sum = __shfl_sync(FULL, sum, 0);
  }
#pragma unroll 1
  for (int e = st; e < NE; e += nst) sp[e] = __double2float_rn(__ddiv_rn(static_cast<double>(sev[e]), sum));
  asm volatile("bar.sync 2, %0;" ::"r"(nst) : "memory");
  if (st >= 32) return;   // the last warp alone from here (st < 32 is the last softmax warp)
  // The true top k lies among the experts whose probability is at least that of the logit order's k-th (probability is
  // monotone in the logit); rank those by (probability down, id up). Candidate c goes to lane c.
  const float pk = sp[m.spec[K - 1]];
  int nc = 0, me = NE;
#pragma unroll 1
  for (int e0 = 0; e0 < NE; e0 += 32) {
    const uint32_t bal = __ballot_sync(FULL, e0 + lane < NE && sp[e0 + lane] >= pk);
    const int cnt = __popc(bal);
    if (me == NE && lane >= nc && lane < nc + cnt) {
      uint32_t m2 = bal;
      for (int t = 0; t < lane - nc; ++t) m2 &= m2 - 1u;
      me = e0 + __ffs(m2) - 1;
    }
    nc += cnt;
  }
  if (nc <= 32) {
    const float mp = me < NE ? sp[me] : -1.f;
    int rank = 0;
    for (int d = 0; d < nc; ++d) {
      const int ed = __shfl_sync(FULL, me, d);
      const float pd = __shfl_sync(FULL, mp, d);
      rank += pd > mp || (pd == mp && ed < me);
    }
    if (lane < nc && rank < K) m.tru[rank] = me;
  } else {
    rank_all_candidates(m, sp, NE, K, pk, lane);
  }
  __syncwarp();
  // weights in rank order (c/src/forward.c:984): every lane forms the same sum by shuffles
  const int ek = lane < K ? m.tru[lane] : -1;
  const float wk = ek >= 0 ? sp[ek] : 0.f;
  float z = 0.f;
  for (int k = 0; k < K; ++k) z = __fadd_rn(z, __shfl_sync(FULL, wk, k));
  const float w = a.norm_topk && z > 0.f ? __fdiv_rn(wk, z) : wk;
  if (lane < K) {
    m.w[lane] = w;
    if (cta0) {
      if (a.sel_out) a.sel_out[lane] = ek;
      if (a.wt_out) a.wt_out[lane] = w;
    }
  }
  __syncwarp();
  // which group streams each true expert (lane k for rank k); a group whose expert is outside the true top k takes a
  // missing one (both in order), so every CTA of that group refetches the same expert
  int gk = -1;
  const int tk = lane < K ? m.tru[lane] : -2;
  for (int h = 0; h < K; ++h) gk = m.spec[h] == tk ? h : gk;
  const int sg = lane < K ? m.spec[lane] : -2;   // lane g: is group g's expert in the true top k?
  bool in = false;
  for (int k = 0; k < K; ++k) in |= m.tru[k] == sg;
  const uint32_t orphan = __ballot_sync(FULL, lane < K && !in), missing = __ballot_sync(FULL, lane < K && gk < 0);
  if (lane < K && gk < 0) {   // the missing rank's position among the missing ranks pairs it with the orphan group at the
                              // same position
    const int pos = __popc(missing & ((1u << lane) - 1u));
    uint32_t o = orphan;
    for (int t = 0; t < pos && o; ++t) o &= o - 1u;
    gk = o ? __ffs(o) - 1 : -1;
    if (gk == kg) m.flag[3] = tk + 1;
  }
  if (lane < K) m.slot[lane] = gk;
  if (lane < K && (gk < 0 || tk < 0)) fail(a, m, ERR_BAD_EXPERT);   // cannot happen: two sets of K experts each
  const uint32_t mine = __ballot_sync(FULL, lane < K && gk == kg);
  if (lane == 0) m.mine = mine ? m.w[__ffs(mine) - 1] : 0.f;
  __syncwarp();
}

}  // namespace
template <uint32_t GT, uint32_t DT>
__global__ void __launch_bounds__(GROUP_THREADS, 1) moe_group_kernel(const GroupArgs a) {
  constexpr int XV = 4096 / 4 / GROUP_THREADS;   // float4 of x per thread (E <= 4096)
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int E = a.E, FF = a.FF, NE = a.NE, K = a.K, ne = a.ne;
  const int nb = E / 256, nbd = FF / 256;
  const bool worker = c < K * ne;
  const int kg = worker ? c / ne : 0, ci = worker ? c - kg * ne : 0;
  const int nre = c < NE ? (NE - c + G - 1) / G : 0;    // experts this CTA scores: c, c + G, ...
  const uint32_t uc = static_cast<uint32_t>(ci), une = static_cast<uint32_t>(ne);
  const int j0 = static_cast<int>(FF * uc / une), j1 = static_cast<int>(FF * (uc + 1) / une);
  const int r0 = static_cast<int>(E * uc / une), r1 = static_cast<int>(E * (uc + 1) / une);
  const int ngu = j1 - j0, nd = r1 - r0;
  const int GL = a.GL, RPW = 32 / GL, nrg = (ngu + RPW - 1) / RPW;
  const int nwg = min(nrg, SW), nbar = 32 * (1 + nwg);   // warps with gate/up rows; the named barrier's threads
  const uint32_t grb = a.grb, drb = a.drb;
  const int PS = E / 8 + 4;   // row stride (floats) of the products: one row per strided chain, rows in different banks

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bars);   // [nrg_max] row groups, [nrg_max] down, [+1] norm/router
  uint64_t *bar_dn = bars + a.nrg_max, *bar_in = bars + a.nrg_max + 1;
  float *sx = reinterpret_cast<float *>(smem + a.off_x);
  float *sw = reinterpret_cast<float *>(smem + a.off_norm);
  float *sxn = reinterpret_cast<float *>(smem + a.off_xn);
  int8_t *xq_qs = reinterpret_cast<int8_t *>(smem + a.off_xq);
  int16_t *xq_bs = reinterpret_cast<int16_t *>(smem + a.off_xq + E);
  float *xq_d = reinterpret_cast<float *>(smem + a.off_xq + E + 2 * (E / 16));
  float *srow = reinterpret_cast<float *>(smem + a.off_router);      // [nre][rstride] router rows
  float *sprod = reinterpret_cast<float *>(smem + a.off_prod);       // [nre][8][PS] products, chain-major
  float *slg = reinterpret_cast<float *>(smem + a.off_lg);            // [NE] logits
  float *sev = reinterpret_cast<float *>(smem + a.off_ev);            // [NE] exponentials
  float *sp = reinterpret_cast<float *>(smem + a.off_p);              // [NE] probabilities
  GroupMisc &m = *reinterpret_cast<GroupMisc *>(smem + a.off_misc);
  float *shg = reinterpret_cast<float *>(smem + a.off_hg);            // [FF] the group's hg
  int8_t *hq_qs = reinterpret_cast<int8_t *>(smem + a.off_hq);
  int16_t *hq_bs = reinterpret_cast<int16_t *>(smem + a.off_hq + FF);
  float *hq_d = reinterpret_cast<float *>(smem + a.off_hq + FF + 2 * (FF / 16));
  float *sterms = reinterpret_cast<float *>(smem + a.off_terms);      // [nd_max][nbd]
  float *sown = reinterpret_cast<float *>(smem + a.off_own);          // [nd_max] this CTA's weighted rows
  float *sgath = reinterpret_cast<float *>(smem + a.off_gath);        // [K][nd_max] the chunk's rows of every group
  uint8_t *sgu = smem + a.off_gu;                                     // [2][nrg_max] regions of rg_bytes
  uint8_t *sdn = smem + a.off_dn;

  trace_time(a.trace, 30);
  trace_stamp(a.trace, 0);
  // ---- 0: barriers; norm weights and router rows (weights only, so before the dependency wait) -----------------------------
  if (tid == 0) {
    for (int s = 0; s < a.nrg_max + 2; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    if (worker || nre > 0) {
      const uint32_t rb = static_cast<uint32_t>(E) * 4u;
      mbar_arrive_expect_tx(bar_in, static_cast<uint32_t>(nre + 1) * rb);
      bulk_copy_g2s(sw, a.norm, rb, bar_in);
      for (int q = 0; q < nre; ++q)
        bulk_copy_g2s(srow + static_cast<size_t>(q) * a.rstride, a.router + static_cast<size_t>(c + q * G) * E, rb, bar_in);
    }
    m.flag[0] = m.flag[1] = m.flag[2] = m.flag[3] = 0;
    m.tiny = 0;
  }
  if (tid <= DECODE_MAX_K) m.spec[tid] = -1;
  if (tid < DECODE_MAX_K) m.tru[tid] = -1;
  __syncthreads();          // the mbarriers are initialised before any thread waits on one
  grid_dependency_wait();   // x and the exchange buffer belong to the previous kernel until here
  grid_launch_dependents();
  const bool active = worker || nre > 0;
  const uint32_t tag = active ? ld_relaxed(a.sync) + 1u : 0u;   // this launch's tag (the previous launch advanced it)

  trace_stamp(a.trace, 1);
  // ---- 1: x, rmsnorm (double sum of squares; c/src/forward.c:412-417), the router products ---------------------------------
  if (active) {
    float4 xv[XV];
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < XV; ++u) {
      const int i = (tid + u * GROUP_THREADS) * 4;
      if (i < E) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x_in + i));
        xv[u] = v;
        reinterpret_cast<float4 *>(sx + i)[0] = v;
        ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
    if (lane == 0) m.red[warp] = ss;
    if (!mbar_wait_bounded(bar_in, 0)) fail(a, m, ERR_WAIT_COPY);
    __syncthreads();
    trace_stamp(a.trace, 2);
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += m.red[w];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / static_cast<double>(E)), a.eps)));
#pragma unroll
    for (int u = 0; u < XV; ++u) {
      const int i = (tid + u * GROUP_THREADS) * 4;
      if (i < E) {
        const float4 v = xv[u], w = reinterpret_cast<const float4 *>(sw + i)[0];
        const float nn[4] = {__fmul_rn(__fmul_rn(v.x, scale), w.x), __fmul_rn(__fmul_rn(v.y, scale), w.y),
                             __fmul_rn(__fmul_rn(v.z, scale), w.z), __fmul_rn(__fmul_rn(v.w, scale), w.w)};
        reinterpret_cast<float4 *>(sxn + i)[0] = make_float4(nn[0], nn[1], nn[2], nn[3]);
#pragma unroll 1
        for (int q = 0; q < nre; ++q) {   // product i goes to chain i % 8, position i / 8
          const float4 r = reinterpret_cast<const float4 *>(srow + static_cast<size_t>(q) * a.rstride + i)[0];
          const float rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) sprod[(q * 8 + ((i + t) & 7)) * PS + ((i + t) >> 3)] = __fmul_rn(rr[t], nn[t]);
        }
      }
    }
    __syncthreads();
  }
  trace_stamp(a.trace, 3);

  // ---- 2: this CTA's logits (the last warp), the Q8_K blocks of xn (the other warps) ---------------------------------------
  if (warp == SW) {
    if (nre > 0) {   // lanes 8q..8q+7 form expert c + q*G (four a pass): lane l8 adds its chain's products in order
      const int grp = lane >> 3, l8 = lane & 7, n4 = E / 32;   // float4 per chain (a multiple of 8)
      for (int q0 = 0; q0 < nre; q0 += 4) {
        const int q = q0 + grp;
        float s = 0.f;
        if (q < nre) {
          const float4 *p4 = reinterpret_cast<const float4 *>(sprod + (q * 8 + l8) * PS);
          float4 v[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) v[t] = p4[t];
          for (int b0 = 0; b0 < n4; b0 += 8) {   // eight float4 in registers while the next eight load
            float4 w[8];
            if (b0 + 8 < n4) {
#pragma unroll
              for (int t = 0; t < 8; ++t) w[t] = p4[b0 + 8 + t];
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[t].x), v[t].y), v[t].z), v[t].w);
            if (b0 + 8 < n4) {
#pragma unroll
              for (int t = 0; t < 8; ++t) v[t] = w[t];
            }
          }
        }
        float p8[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) p8[l] = __shfl_sync(FULL, s, (lane & ~7) + l);
        if (q < nre && l8 == 0) {
          const float lg = __fadd_rn(__fadd_rn(__fadd_rn(p8[0], p8[1]), __fadd_rn(p8[2], p8[3])),
                                     __fadd_rn(__fadd_rn(p8[4], p8[5]), __fadd_rn(p8[6], p8[7])));
          st_word(a.lw + c + q * G, tag, fbits(lg));
        }
      }
      if (lane == 0) trace_stamp_here(a.trace, 4);
    }
  } else if (worker) {
    // the warps of the three SM sub-partitions without the scoring warp (a warp's sub-partition is its index mod 4), so
    // none competes with its chains for issue slots
    if ((warp & 3) != (SW & 3))
      q8k_blocks(sxn, E, xq_qs, xq_d, xq_bs, (warp >> 2) * 3 + ((warp & 3) < (SW & 3) ? (warp & 3) : (warp & 3) - 1), NW / 4 * 3, lane);
  }
  if (!worker) goto done;   // a CTA that only scores experts is finished

  // ---- 3: every logit, the ranking by logit (ties to the lower id) ---------------------------------------------------------
  if (!gather_words([&](int i) { return a.lw + i; }, [&](int i) { return slg + i; }, NE, tag, tid, GROUP_THREADS))
    fail(a, m, ERR_WAIT_ROUTER);
  if (tid < ((NE + 3) & ~3) - NE) slg[NE + tid] = -INFINITY;
  trace_stamp(a.trace, 21);
  __syncthreads();
  trace_stamp(a.trace, 5);
  if (!m.flag[0]) {
    // rank = the experts ahead of e in the order (logit down, id up): four threads per expert, each a quarter of the
    // rivals by broadcast float4 loads (the logits past NE read as -inf)
    const int n4 = (NE + 3) / 4, per = (n4 + 3) / 4;
#pragma unroll 1
    for (int e0 = 0; e0 < NE; e0 += GROUP_THREADS / 4) {
      const int e = e0 + (tid >> 2), part = tid & 3;
      const float le = e < NE ? slg[e] : 0.f;
      const float4 *l4 = reinterpret_cast<const float4 *>(slg);
      int rank = 0;
#pragma unroll 1
      for (int u = 0; u < per; ++u) {
        const int q = part * per + u;
        if (q < n4) {
          const float4 v = l4[q];
          const int f = 4 * q;
          rank += (v.x > le || (v.x == le && f < e)) + (v.y > le || (v.y == le && f + 1 < e)) +
                  (v.z > le || (v.z == le && f + 2 < e)) + (v.w > le || (v.w == le && f + 3 < e));
        }
      }
      rank += __shfl_xor_sync(FULL, rank, 1);
      rank += __shfl_xor_sync(FULL, rank, 2);
      if (e < NE && part == 0) {
        if (rank <= K) m.spec[rank] = e;
        if (rank == 0) m.top = e;
      }
    }
  }
  trace_stamp(a.trace, 22);
  __syncthreads();
  trace_stamp(a.trace, 23);
  if (tid == 0 && !m.flag[0]) {
    for (int k = 0; k < K; ++k)
      if (m.spec[k] < 0) fail(a, m, ERR_BAD_EXPERT);   // logits that do not order (NaN)
    if (!m.flag[0] && a.force_miss && K < NE) { const int t = m.spec[K - 1]; m.spec[K - 1] = m.spec[K]; m.spec[K] = t; }
  }
  __syncthreads();
  trace_stamp(a.trace, 6);

  {
    // ---- 4: the copies of this CTA's rows of its group's expert ------------------------------------------------------------
    auto src = [&](int e, int q, int row) -> const uint8_t * {   // q: 0 gate, 1 up, 2 down
      const size_t ee = static_cast<size_t>(e);
      return q == 0 ? a.gate + ee * a.gate_slab + static_cast<size_t>(row) * grb
           : q == 1 ? a.up + ee * a.up_slab + static_cast<size_t>(row) * grb
                    : a.down + ee * a.down_slab + static_cast<size_t>(row) * drb;
    };
    auto issue = [&](int e) {   // lane 0 of warp w: row groups w, w + NW, ...; lane 0 of the last warp also the down rows
      if (lane != 0) return;
#pragma unroll 1
      for (int g = warp; g < nrg; g += NW) {
        const int ra = j0 + g * RPW, rb = min(j1, ra + RPW);
        const uint32_t len = static_cast<uint32_t>(rb - ra) * grb;
        const uint8_t *s0 = src(e, 0, ra), *s1 = src(e, 1, ra);
        const uint32_t lo0 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s0) & 15u),
                       lo1 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s1) & 15u);
        const uint32_t n0 = (lo0 + len + 15u) & ~15u, n1 = (lo1 + len + 15u) & ~15u;
        mbar_arrive_expect_tx(&bars[g], n0 + n1);
        bulk_copy_g2s(sgu + static_cast<size_t>(g) * a.rg_bytes, s0 - lo0, n0, &bars[g]);
        bulk_copy_g2s(sgu + static_cast<size_t>(a.nrg_max + g) * a.rg_bytes, s1 - lo1, n1, &bars[g]);
      }
      if (warp == NW - 1) {
        const uint8_t *s2 = src(e, 2, r0);
        const uint32_t lo2 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s2) & 15u);
        const uint32_t n2 = (lo2 + static_cast<uint32_t>(nd) * drb + 15u) & ~15u;
        mbar_arrive_expect_tx(bar_dn, n2);
        bulk_copy_g2s(sdn, s2 - lo2, n2, bar_dn);
      }
    };
    if (tid == 0 && !m.flag[0] && (m.top < 0 || m.top >= NE || m.spec[kg] < 0 || m.spec[kg] >= NE)) fail(a, m, ERR_BAD_EXPERT);
    __syncthreads();
    const bool go = !m.flag[0];   // uniform: read after a block barrier
    int e_mine = m.spec[kg];
    uint32_t ph = 0;
    // ---- 5 and 6: the softmax warp's verdict; the gate/up rows on the other warps. Round 0 works on the logit order's
    // expert; a second round (rare: this group's expert is not in the true top k) waits for the first copies, fetches the
    // right expert and redoes the rows. One copy of the code serves both rounds.
    for (int round = 0; go; ++round) {
      if (round == 1) {
        if (tid == 0) {
          for (int g = 0; g < nrg; ++g) if (!mbar_wait_bounded(&bars[g], 0)) fail(a, m, ERR_WAIT_COPY);
          if (!mbar_wait_bounded(bar_dn, 0)) fail(a, m, ERR_WAIT_COPY);
          m.flag[3] = 0;
        }
        __syncthreads();
        for (int k = 0; k < K; ++k) if (m.slot[k] == kg) e_mine = m.tru[k];
        fence_proxy_async();   // the generic reads of the slots before the async copies rewrite them
        ph = 1;
      }
      issue(e_mine);
      if (round == 0) trace_stamp(a.trace, 24);
      if (tid == 0) m.flag[1] = round + 1;
      if (round == 0) trace_stamp(a.trace, 7);
      if (warp >= nwg) {   // the softmax warps; the last one hands the verdict to the gate/up warps
        if (round == 0) {
          softmax_verdict(a, m, slg, sev, sp, kg, (SW - warp) * 32 + lane, (NW - nwg) * 32, c == 0);
          if (warp == SW && lane == 0) trace_stamp_here(a.trace, 28);
          if (warp == SW) named_arrive(nbar);
        }
      } else {   // row groups warp, warp + SW, ...
        const int lg = lane & (GL - 1), rw = lane / GL, base = lane - lg;
        const bool has_blk = lg < nb;
        BlockAct act;
        if (has_blk) load_block_act(xq_qs, xq_d, xq_bs, lg, act);
        bool synced = round > 0;
#pragma unroll 1
        for (int g = warp; g < nrg; g += SW) {   // the same trip count in every lane of a warp
          if (!mbar_wait_bounded(&bars[g], ph)) fail(a, m, ERR_WAIT_COPY);
          if (g == 0 && round == 0) trace_stamp(a.trace, 25);
          const int j = j0 + g * RPW + rw;
          const bool valid = j < j1;
          float tg = 0.f, tu = 0.f;
          if (valid && has_blk) {
            const uint32_t lo0 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src(e_mine, 0, j0 + g * RPW)) & 15u);
            const uint32_t lo1 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src(e_mine, 1, j0 + g * RPW)) & 15u);
            const uint8_t *rg0 = sgu + static_cast<size_t>(g) * a.rg_bytes + lo0 + static_cast<size_t>(rw) * grb;
            const uint8_t *rg1 = sgu + static_cast<size_t>(a.nrg_max + g) * a.rg_bytes + lo1 + static_cast<size_t>(rw) * grb;
#pragma unroll 1
            for (int q = 0; q < 2; ++q) {   // one copy of the block code
              const float t = kq_block(GT, q == 0 ? rg0 : rg1, lg, act);
              if (q == 0) tg = t; else tu = t;
            }
          }
          float sg = 0.f, su = 0.f;   // the row's block terms in block order
#pragma unroll 1
          for (int b = 0; b < nb; ++b) {
            sg = __fadd_rn(sg, __shfl_sync(FULL, tg, base + b));
            su = __fadd_rn(su, __shfl_sync(FULL, tu, base + b));
          }
          if (!synced) { named_sync(nbar); synced = true; if (round == 0) trace_stamp(a.trace, 26); }   // the verdict first
          if (valid && lg == 0 && !m.flag[3]) st_word(a.hw + static_cast<size_t>(kg) * FF + j, tag, fbits(silu_mul(sg, su)));
        }
      }
      if (round == 0) trace_stamp(a.trace, 27);
      __syncthreads();
      if (round == 0) trace_stamp(a.trace, 8);
      if (round > 0 || !m.flag[3]) break;   // uniform: read after the barrier
    }
    trace_stamp(a.trace, 9);

    // ---- 7: the group's hg, its Q8_K blocks, the down rows' terms, wt * hd -----------------------------------------------
    if (!m.flag[0]) {
      const unsigned long long *hwk = a.hw + static_cast<size_t>(kg) * FF;
      if (!gather_words([&](int i) { return hwk + i; }, [&](int i) { return shg + i; }, FF, tag, tid, GROUP_THREADS))
        fail(a, m, ERR_WAIT_EXPERT);
      __syncthreads();
      trace_stamp(a.trace, 10);
    }
    if (!m.flag[0]) {
      q8k_blocks(shg, FF, hq_qs, hq_d, hq_bs, warp, NW, lane);
      if (!mbar_wait_bounded(bar_dn, ph)) fail(a, m, ERR_WAIT_COPY);
      __syncthreads();
      trace_stamp(a.trace, 11);
    }
    if (!m.flag[0]) {
      const uint32_t lo2 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src(e_mine, 2, r0)) & 15u);
#pragma unroll 1
      for (int t0 = 0; t0 < nd * nbd; t0 += GROUP_THREADS) {   // block-major: a warp's lanes mostly share one activation block
        const int t = t0 + tid;
        const int b = min(t / nd, nbd - 1), r = t - b * nd;
        BlockAct act;
        load_block_act(hq_qs, hq_d, hq_bs, b, act);
        if (t < nd * nbd) sterms[r * nbd + b] = kq_block(DT, sdn + lo2 + static_cast<size_t>(r) * drb, b, act);
      }
      __syncthreads();
      trace_stamp(a.trace, 12);
      const float wk = m.mine;
      const bool combiner = kg == ci % K;
#pragma unroll 1
      for (int r = tid; r < nd; r += GROUP_THREADS) {
        float hd = 0.f;
#pragma unroll 1
        for (int b = 0; b < nbd; ++b) hd = __fadd_rn(hd, sterms[r * nbd + b]);
        const float v = __fmul_rn(wk, hd);
        if (combiner) sown[r] = v;
        else st_word(a.hw + static_cast<size_t>(K) * FF + static_cast<size_t>(kg) * E + r0 + r, tag, fbits(v));
      }
      trace_stamp(a.trace, 13);
      // ---- 8: the chunk's combine in rank order and the residual (c/src/forward.c:1026-1032) ---------------------------------
      if (combiner) {
        const unsigned long long *wpw = a.hw + static_cast<size_t>(K) * FF;   // the weighted rows' words follow the hg words
        // the other groups' words of the chunk, all in one pass (this CTA's own rows are in sown): index i -> group g of the
        // K - 1 others, row r
        const int nd_ = nd, kg_ = kg, ndm = a.nd_max;
        auto wa = [&](int i) { const int q = i / nd_, g = q + (q >= kg_); return wpw + static_cast<size_t>(g) * E + r0 + (i - q * nd_); };
        auto wd = [&](int i) { const int q = i / nd_, g = q + (q >= kg_); return sgath + g * ndm + (i - q * nd_); };
        if (!gather_words(wa, wd, (K - 1) * nd, tag, tid, GROUP_THREADS)) fail(a, m, ERR_WAIT_EXPERT);
        __syncthreads();
        if (!m.flag[0]) {
#pragma unroll 1
          for (int r = tid; r < nd; r += GROUP_THREADS) {
            float moe = 0.f;
#pragma unroll 1
            for (int k = 0; k < K; ++k) {
              const int g = m.slot[k];
              if (g < 0 || g >= K) { fail(a, m, ERR_BAD_EXPERT); break; }
              moe = __fadd_rn(moe, g == kg ? sown[r] : sgath[g * a.nd_max + r]);
            }
            a.x_out[r0 + r] = __fadd_rn(sx[r0 + r], __fmul_rn(a.resid_scale, moe));
          }
        }
        if (c == 0 && tid == 0) {   // every CTA that reads the generation has read it: its words reached this combine
          __threadfence();
          atomicExch(a.sync, tag);
          m.flag[2] = 1;
        }
      }
    }
  }

done:
  // ---- exit: copies in flight land first -------------------------------------------------------------------------------------
  __syncthreads();
  trace_stamp(a.trace, 19);
  trace_time(a.trace, 31);
  if (tid == 0 && m.flag[1] && m.flag[0]) {   // an error path may leave copies unwaited
    const uint32_t ph = static_cast<uint32_t>(m.flag[1] - 1);
    for (int g = 0; g < nrg; ++g) mbar_wait_bounded(&bars[g], ph);
    mbar_wait_bounded(bar_dn, ph);
  }
  if (c == 0 && tid == 0 && active && !m.flag[2]) {   // a failed launch still moves the generation on (the host, told of the
    __threadfence();                                   // failure, clears the exchange buffer before the next call)
    atomicExch(a.sync, tag);
  }
}

size_t group_buffer_bytes(int sms, int E, int FF, int NE, int K) {
  const size_t head = (static_cast<size_t>(2 + sms) * 4 + 255) / 256 * 256;
  return head + (static_cast<size_t>(NE) * 8 + 255) / 256 * 256 + static_cast<size_t>(K) * (FF + E) * 8;
}

void group_set_buffer(GroupArgs &a, uint8_t *buf, int sms) {
  const size_t head = (static_cast<size_t>(2 + sms) * 4 + 255) / 256 * 256;
  const size_t lwb = (static_cast<size_t>(a.NE) * 8 + 255) / 256 * 256;
  a.sync = reinterpret_cast<uint32_t *>(buf);
  a.lw = reinterpret_cast<unsigned long long *>(buf + head);
  a.hw = reinterpret_cast<unsigned long long *>(buf + head + lwb);
}

int plan_group_shape(int sms, int max_smem, int E, int FF, int NE, int K, uint32_t gate_type, uint32_t up_type,
                     uint32_t down_type, GroupArgs &a) {
  auto kq = [](uint32_t t) { return t == T_Q4_K || t == T_Q6_K; };
  if (!kq(gate_type) || gate_type != up_type || !kq(down_type)) return 1;
  if (E < 256 || E % 256 || E > 4096 || FF < 256 || FF % 256 || FF > 4096) return 1;
  if (K < 1 || K > DECODE_MAX_K || NE < K || NE > GROUP_MAX_NE || sms < K) return 1;
  const int ne = sms / K, nre = (NE + sms - 1) / sms;
  if (nre > 4) return 1;
  const int nb = E / 256, nbd = FF / 256;
  const int GL = nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : nb <= 8 ? 8 : 16;
  const int RPW = 32 / GL;
  a.ne = ne;
  a.GL = GL;
  a.nre = nre;
  a.ngu_max = (FF + ne - 1) / ne;
  a.nd_max = (E + ne - 1) / ne;
  a.nrg_max = (a.ngu_max + RPW - 1) / RPW;
  if (a.nrg_max > GROUP_MAX_RG) return 1;
  if (static_cast<size_t>(a.nd_max) * nbd > 4 * static_cast<size_t>(GROUP_THREADS)) return 1;
  auto rowb = [](uint32_t t, int n) { return static_cast<uint32_t>(t == T_Q4_K ? n / 256 * 144 : n / 256 * 210); };
  a.grb = rowb(gate_type, E);
  a.drb = rowb(down_type, FF);
  a.rg_bytes = (static_cast<uint32_t>(RPW) * a.grb + 32u + 15u) & ~15u;
  a.rstride = static_cast<uint32_t>(E + 8);
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = (o + bytes + 15) / 16 * 16; return static_cast<uint32_t>(at); };
  a.off_bars = take(8 * (a.nrg_max + 2));
  a.off_misc = take(sizeof(GroupMisc));
  a.off_x = take(static_cast<size_t>(E) * 4);
  a.off_norm = take(static_cast<size_t>(E) * 4);
  a.off_xn = take(static_cast<size_t>(E) * 4);
  a.off_xq = take(static_cast<size_t>(E) + 2 * (E / 16) + 4 * (E / 256));
  a.off_lg = take(static_cast<size_t>(NE) * 4);
  a.off_ev = take(static_cast<size_t>(NE) * 4);
  a.off_p = take(static_cast<size_t>(NE) * 4);
  a.off_hg = take(static_cast<size_t>(FF) * 4);
  a.off_hq = take(static_cast<size_t>(FF) + 2 * (FF / 16) + 4 * (FF / 256));
  a.off_terms = take(static_cast<size_t>(a.nd_max) * nbd * 4);
  a.off_router = take(static_cast<size_t>(nre) * a.rstride * 4);
  a.off_prod = take(static_cast<size_t>(nre) * 8 * (E / 8 + 4) * 4);
  a.off_own = take(static_cast<size_t>(a.nd_max) * 4);
  a.off_gath = take(static_cast<size_t>(K) * a.nd_max * 4);
  o = (o + 127) / 128 * 128;
  a.off_gu = take(2 * static_cast<size_t>(a.nrg_max) * a.rg_bytes);
  a.off_dn = take(static_cast<size_t>(a.nd_max) * a.drb + 32);
  const size_t total = o + 16;
  if (total > static_cast<size_t>(max_smem)) return 1;
  a.smem_bytes = static_cast<uint32_t>(total);
  return 0;
}

GroupFn group_kernel_for(uint32_t gate_type, uint32_t down_type) {
  if (gate_type == T_Q4_K) return down_type == T_Q4_K ? moe_group_kernel<T_Q4_K, T_Q4_K> : down_type == T_Q6_K ? moe_group_kernel<T_Q4_K, T_Q6_K> : nullptr;
  if (gate_type == T_Q6_K) return down_type == T_Q4_K ? moe_group_kernel<T_Q6_K, T_Q4_K> : down_type == T_Q6_K ? moe_group_kernel<T_Q6_K, T_Q6_K> : nullptr;
  return nullptr;
}

cudaError_t group_allow_smem(int bytes) {
  const GroupFn fns[4] = {moe_group_kernel<T_Q4_K, T_Q4_K>, moe_group_kernel<T_Q4_K, T_Q6_K>, moe_group_kernel<T_Q6_K, T_Q4_K>,
                          moe_group_kernel<T_Q6_K, T_Q6_K>};
  for (GroupFn f : fns) {
    const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace clb
