// The one-token MoE block as one persistent kernel: the reference's c/src/forward.c:949-1033 on one B200.
//
// Modes (DecodeArgs::mode): 0 runs every phase below; 1 stops after phase 3 (routing only, for a host that must see the
// choice before it places the experts -- the expert store); 2 skips the router (phases 2-3) and takes the routing and the
// experts' addresses from its arguments (the experts as the store placed them in HBM).
//
// One CTA per SM (G CTAs, all co-resident), 512 threads. Every CTA streams the same share of every chosen expert, and all
// of a CTA's share of the chosen experts sits in shared memory at once. Data that crosses CTAs goes through global memory
// behind two counters (bounded waits). The phases are laid out for latency: at one token nearly all of the time is
// dependent steps, not bytes, so each step runs on as few block-wide barriers as it can.
//   0  (before the programmatic-launch wait, overlapping the previous kernel's tail) barriers; this CTA's router rows
//      (experts c, c+G, ...) and the norm weights start streaming into shared memory;
//   1  x (in registers), the double sum of squares, xn = rmsnorm(x) (c/src/forward.c:412-417);
//   2  the last warp forms this CTA's router logits as the reference's dotf does (c/src/forward.c:574-581): eight lanes per
//      expert, eight strided float sums in element order, combined ((0+1)+(2+3))+((4+5)+(6+7)); logits to global memory,
//      counter 0 += experts scored. Meanwhile the warps of the other SM sub-partitions form the Q8_K blocks of xn;
//      In mode 1 with router-ahead, the next layer's norm and router rows stream into the free expert slots too, and the
//      idle warp of the router warp's sub-partition forms the next layer's logits on this x the same way (counter 0 then
//      counts 2 NE); CTA 0 ranks them after phase 3 (c/src/forward.c:937-946);
//   3  when counter 0 reaches NE, DECODE_THREADS / 4 threads form the softmax, one expert each (double sum,
//      c/src/forward.c:954-958); every thread then ranks a quarter of an expert's competitors (ties to the lower id: the
//      order of the reference's repeated arg-max, c/src/forward.c:975-980); warp 0 renormalises (c/src/forward.c:984).
//      Every CTA does this itself;
//   4  one lane per chosen expert issues the bulk copies of this CTA's share of it: gate and up rows [FF*c/G, FF*(c+1)/G),
//      down rows [E*c/G, E*(c+1)/G);
//   5  a group of lanes per (expert, row): one lane per 256-element block (exact integer sums, the reference's float block
//      term) for the gate row and the up row, the terms added in block order across the group by shuffles, SwiGLU
//      (c/src/forward.c:1018) at the group's first lane, hg to global memory; counter 1 += 1 per CTA;
//   6  when counter 1 reaches G: the Q8_K blocks of every expert's hg; down rows (same arithmetic; a group of lanes per
//      (expert, block), one row each); wt * hd per (row, expert), then per output row moe = their sum in rank order;
//      x = x + resid_scale * moe; the last CTA out resets the counters.
#include "common.cuh"
#include "decode.cuh"
#include "route.cuh"
#include "rowdot.cuh"

namespace clb {

// GT: the gate and up experts' type, DT: the down experts' type (Q4_K or Q6_K each): one instantiation per pair keeps the
// code a launch runs small enough to stay in the instruction caches from one layer's launch to the next.
template <uint32_t GT, uint32_t DT>
__global__ void __launch_bounds__(DECODE_THREADS, 1) moe_decode_kernel(const DecodeArgs a) {
  constexpr int NW = DECODE_THREADS / 32;
  constexpr int RW = NW - 1;                           // the router warp
  constexpr int XV = 4096 / 4 / DECODE_THREADS;        // float4 of x per thread (E <= 4096)
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int E = a.E, FF = a.FF, NE = a.NE, K = a.K;
  const int nb = E / 256, nbd = FF / 256;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bars);   // [K] slots' gate/up rows, [K] router rows + norm weights
  uint64_t *dbar = bars + K + 1;                                       // [K] slots' down rows
  float *xn = reinterpret_cast<float *>(smem + a.off_xn);             // [E] xn
  float *wn = reinterpret_cast<float *>(smem + a.off_norm);           // [E] norm weights
  int8_t *xq_qs = reinterpret_cast<int8_t *>(smem + a.off_xq);        // Q8_K of xn: qs [E], bsums [E/16], d [E/256]
  int16_t *xq_bs = reinterpret_cast<int16_t *>(smem + a.off_xq + E);
  float *xq_d = reinterpret_cast<float *>(smem + a.off_xq + E + 2 * (E / 16));
  float *rrows = reinterpret_cast<float *>(smem + a.off_router);      // [nre][E] router rows
  float *rprod = reinterpret_cast<float *>(smem + a.off_rprod);       // [nre][8][E/8 + 4]: product i in row i % 8, column i / 8
  double *s_red = reinterpret_cast<double *>(smem + a.off_misc);      // [NW]
  int *s_flag = reinterpret_cast<int *>(s_red + NW);                   // [0] failed, [2] probability order differs
  int *s_sel = s_flag + 4;                                             // [32] chosen experts, rank order
  float *s_wt = reinterpret_cast<float *>(s_sel + 32);                 // [32] their router probabilities
  float *s_wn = s_wt + 32;                                             // [32] the weights the combine uses
  float *probs = s_wn + 32;                                            // [DECODE_THREADS / 4]
  float *s_lg = probs + DECODE_THREADS / 4;                            // [DECODE_THREADS / 4] logits, -inf past NE
  int *s_spec = reinterpret_cast<int *>(s_lg + DECODE_THREADS / 4);   // [DECODE_MAX_K + 1] slot k: the expert it streams
  int *s_slot = s_spec + DECODE_MAX_K + 4;                             // [K] rank -> the slot streaming that expert
  int *s_par = s_slot + DECODE_MAX_K;                                  // [K] parity of the phase the slot's copies complete
  int *s_iss = s_par + DECODE_MAX_K;                                   // [K] copies issued into the slot: 1 gate/up, 2 down
  int *s_fix = s_iss + DECODE_MAX_K;                                   // [K] expert + 1 to fetch into the slot again, or 0
  float *terms = reinterpret_cast<float *>(smem + a.off_terms);       // block terms of the down rows
  int8_t *hq_qs = reinterpret_cast<int8_t *>(smem + a.off_hq);        // Q8_K of every expert's hg: qs [K*FF], bsums, d
  int16_t *hq_bs = reinterpret_cast<int16_t *>(smem + a.off_hq + K * FF);
  float *hq_d = reinterpret_cast<float *>(smem + a.off_hq + K * FF + 2 * (K * FF / 16));
  float *xr = reinterpret_cast<float *>(smem + a.off_xr);             // [rd_max] this CTA's rows of x
  uint8_t *slots = smem + a.off_slots;

  const uint32_t uG = static_cast<uint32_t>(G), uc = static_cast<uint32_t>(c);   // FF, E <= 4096: the products fit 32 bits
  const int j0 = static_cast<int>(FF * uc / uG), j1 = static_cast<int>(FF * (uc + 1) / uG);
  const int i0 = static_cast<int>(E * uc / uG), i1 = static_cast<int>(E * (uc + 1) / uG);
  const int ngu = j1 - j0, nd = i1 - i0;
  const int nre = (a.mode != 2 && c < NE) ? (NE - c + G - 1) / G : 0;   // experts this CTA scores: c, c+G, ...
  const uint32_t grb = a.grb, drb = a.drb, gseg = a.gseg;
  const int RS = E / 8 + 4;   // row stride of rprod (floats): the eight rows start in different banks
  // router-ahead (mode 1 only): the next layer's norm weights, router rows, products and logits in the expert slots
  const bool ahead = a.mode == 1 && a.ahead_n > 0;
  float *wn2 = reinterpret_cast<float *>(slots);
  float *rrows2 = wn2 + E;
  float *rprod2 = rrows2 + static_cast<size_t>(nre) * E;
  float *lg2 = rprod2 + static_cast<size_t>(nre) * 8 * RS;

  trace_time(a.trace, 30);
  trace_stamp(a.trace, 0);
  // ---- 0: barriers, router rows and norm weights (weights only, so before the dependency wait) ------------------------------
  if (tid == 0) {
    for (int s = 0; s <= 2 * K; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bars[K], static_cast<uint32_t>(nre + 1) * E * 4u * (ahead ? 2u : 1u));
    bulk_copy_g2s(wn, a.norm, E * 4u, &bars[K]);
    for (int m = 0; m < nre; ++m)
      bulk_copy_g2s(rrows + static_cast<size_t>(m) * E, a.router + static_cast<size_t>(c + m * G) * E, E * 4u, &bars[K]);
    if (ahead) {
      bulk_copy_g2s(wn2, a.ahead_norm, E * 4u, &bars[K]);
      for (int m = 0; m < nre; ++m)
        bulk_copy_g2s(rrows2 + static_cast<size_t>(m) * E, a.ahead_router + static_cast<size_t>(c + m * G) * E, E * 4u, &bars[K]);
    }
    s_flag[0] = 0;
    s_flag[2] = 0;
  }
  __syncthreads();          // the mbarriers are initialised before any thread waits on one
  grid_dependency_wait();   // x, the scratch and the counters belong to the previous kernel until here
  grid_launch_dependents();

  trace_stamp(a.trace, 1);
  // ---- 1: rmsnorm (double sum of squares; c/src/forward.c:412-417), x kept in registers ----------------------------------
  {
    float4 xv[XV];
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < XV; ++u) {
      const int i = (tid + u * DECODE_THREADS) * 4;
      if (i < E) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x_in + i));
        xv[u] = v;
        ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
    if (lane == 0) s_red[warp] = ss;
    trace_stamp(a.trace, 2);
    if (!mbar_wait_bounded(&bars[K], 0)) set_error(a.err, ERR_WAIT_COPY);
    __syncthreads();
    trace_stamp(a.trace, 3);
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += s_red[w];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / static_cast<double>(E)), a.eps)));
#pragma unroll
    for (int u = 0; u < XV; ++u) {
      const int i = (tid + u * DECODE_THREADS) * 4;
      if (i < E) {
        const float4 v = xv[u], w = reinterpret_cast<const float4 *>(wn + i)[0];
        const float vv[4] = {v.x, v.y, v.z, v.w}, nn[4] = {__fmul_rn(__fmul_rn(v.x, scale), w.x), __fmul_rn(__fmul_rn(v.y, scale), w.y),
                                                           __fmul_rn(__fmul_rn(v.z, scale), w.z), __fmul_rn(__fmul_rn(v.w, scale), w.w)};
        reinterpret_cast<float4 *>(xn + i)[0] = make_float4(nn[0], nn[1], nn[2], nn[3]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (i + q >= i0 && i + q < i1) xr[i + q - i0] = vv[q];
        for (int m = 0; m < nre; ++m)   // the router products, laid out for the strided sums of phase 2
#pragma unroll
          for (int q = 0; q < 4; ++q) rprod[(m * 8 + ((i + q) & 7)) * RS + ((i + q) >> 3)] = __fmul_rn(rrows[m * E + i + q], nn[q]);
        if (ahead) {   // the next layer's rmsnorm of the same x (the same scale), and its router products
          const float4 w2 = reinterpret_cast<const float4 *>(wn2 + i)[0];
          const float n2[4] = {__fmul_rn(__fmul_rn(v.x, scale), w2.x), __fmul_rn(__fmul_rn(v.y, scale), w2.y),
                               __fmul_rn(__fmul_rn(v.z, scale), w2.z), __fmul_rn(__fmul_rn(v.w, scale), w2.w)};
          for (int m = 0; m < nre; ++m)
#pragma unroll
            for (int q = 0; q < 4; ++q) rprod2[(m * 8 + ((i + q) & 7)) * RS + ((i + q) >> 3)] = __fmul_rn(rrows2[m * E + i + q], n2[q]);
        }
      }
    }
    __syncthreads();
  }

  trace_stamp(a.trace, 4);
  // ---- 2: this CTA's router logits (last warp), the Q8_K blocks of xn (the other warps) ------------------------------------
  // one warp forms this CTA's logits from a product buffer: eight lanes per expert, four experts per pass
  auto score = [&](const float *prod, float *out, bool stamp) {
    const int grp = lane >> 3, l8 = lane & 7;
    for (int m0 = 0; m0 < nre; m0 += 4) {   // four experts per pass, eight lanes each
      const int m = m0 + grp;
      float s = 0.f;
      if (m < nre) {   // lane l8 adds products l8, l8 + 8, l8 + 16, ... in order: its row of the products, four float4 at a
                       // time, the next four loaded while these are added (E / 32, the float4 per lane, is a multiple of 8)
        const float4 *p4 = reinterpret_cast<const float4 *>(prod + (m * 8 + l8) * RS);
        float4 v[4], w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = w[t] = p4[t];
        for (int q = 0; q < E / 32; q += 4) {
          if (q + 4 < E / 32) {
#pragma unroll
            for (int t = 0; t < 4; ++t) w[t] = p4[q + 4 + t];
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[t].x), v[t].y), v[t].z), v[t].w);
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = w[t];
        }
      }
      if (stamp && lane == 0 && m0 == 0) trace_stamp_here(a.trace, 24);
      float p8[8];
#pragma unroll
      for (int l = 0; l < 8; ++l) p8[l] = __shfl_sync(FULL, s, (lane & ~7) + l);
      if (m < nre && l8 == 0)
        out[c + m * G] = __fadd_rn(__fadd_rn(__fadd_rn(p8[0], p8[1]), __fadd_rn(p8[2], p8[3])),
                                   __fadd_rn(__fadd_rn(p8[4], p8[5]), __fadd_rn(p8[6], p8[7])));
    }
    __syncwarp();
    if (lane == 0) red_release_add(&a.sync[0], static_cast<uint32_t>(nre));   // release: the warp's logits, ordered by bar.warp.sync
  };
  if (warp == RW) {
    if (nre > 0) {
      score(rprod, a.logits, true);
      if (lane == 0) trace_stamp_here(a.trace, 5);
    }
  } else if (warp == RW - 4 && ahead) {   // idle in mode 1: the router warp's sub-partition, the next layer's logits
    if (nre > 0) score(rprod2, a.logits + NE, false);
  } else if ((warp & 3) != (RW & 3)) {
    // the warps of the other three SM sub-partitions form the Q8_K blocks of xn, so none competes with the router warp's
    // chains for issue slots (a warp's sub-partition is its index mod 4)
    const int qw = (warp >> 2) * 3 + ((warp & 3) < (RW & 3) ? (warp & 3) : (warp & 3) - 1);
    q8k_quantize_block(xn, E, xq_qs, xq_d, xq_bs, qw, NW / 4 * 3, lane, true);
    trace_stamp(a.trace, 6);
  }

  // ---- 3: routing (c/src/forward.c:954-984). Mode 0 ranks the experts by logit first and sends the expert copies out on
  // that order at once: softmax is monotone, so it is the probability order except where two different logits round to
  // the same probability. The softmax, the probability order and the weights follow while the copies fly; a slot whose
  // expert turns out not to be chosen (a probability tie at rank K) fetches the missing one. -----------------------------
  const bool spec = a.mode == 0;
  if (a.mode == 2) {   // the routing is given, renormalised already
    if (tid < K) {
      const int e = a.sel_in[tid];
      if (e < 0 || e >= NE) { set_error(a.err, ERR_BAD_EXPERT); s_flag[0] = 1; }
      s_sel[tid] = e;
      s_wt[tid] = a.wt_in[tid];
      s_wn[tid] = a.wt_in[tid];
      s_spec[tid] = e;
      s_slot[tid] = tid;
    }
  } else if (tid == 0 && !(a.stall_wait ? wait_counter(&a.sync[0], static_cast<uint32_t>(NE) + 1u, a.stall_wait)
                                         : wait_counter(&a.sync[0], static_cast<uint32_t>(NE) * (ahead ? 2u : 1u)))) {
    set_error(a.err, ERR_WAIT_ROUTER);
    s_flag[0] = 1;
  }
  if (tid < DECODE_MAX_K) { s_par[tid] = 0; s_iss[tid] = 0; s_fix[tid] = 0; }
  if (a.mode != 2 && tid < DECODE_MAX_K) s_sel[tid] = -1;
  if (spec && tid <= DECODE_MAX_K) s_spec[tid] = -1;
  __syncthreads();
  trace_stamp(a.trace, 7);
  constexpr int SW = DECODE_THREADS / 4 / 32;   // softmax warps, one expert per thread
  float lv = -INFINITY, mx = -INFINITY, ev = 0.f;
  if (a.mode != 2 && !s_flag[0]) {
    lv = tid < NE ? __ldcg(a.logits + tid) : -INFINITY;
    mx = lv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0 && warp < SW) s_wt[warp] = mx;   // s_wt is written after the ranking
    // NaN ranks as -inf here, so the ranks by logit are a permutation and every slot gets one expert (a NaN routing then
    // fails in the probability check below, with every copy accounted for)
    if (spec && tid < DECODE_THREADS / 4) s_lg[tid] = lv == lv ? lv : -INFINITY;
  }
  __syncthreads();
  trace_stamp(a.trace, 8);
  if (a.mode != 2 && !s_flag[0]) {
    mx = s_wt[0];
#pragma unroll
    for (int w = 1; w < SW; ++w) mx = fmaxf(mx, s_wt[w]);
  }
  // rank of expert tid / 4 = experts ahead of it in the reference's arg-max order (ties to the lower id), counted by four
  // threads over every fourth float4 of the values each (so the four read different banks; v padded with `pad`, below
  // every value, to a multiple of 4)
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
  int my_rank = DECODE_MAX_K + 1;   // spec path: this thread's expert's rank by logit, if it owns one (tid % 4 == 0)
  if (spec && !s_flag[0]) {   // the logit order through rank K
    int rank = rank4(s_lg, -INFINITY);
    if (a.force_miss && K < NE) rank = rank == K - 1 ? K : rank == K ? K - 1 : rank;   // test hook: ranks K - 1 and K swap
    if ((tid >> 2) < NE && (tid & 3) == 0 && rank <= K) {
      s_spec[rank] = tid >> 2;
      my_rank = rank;
    }
  }
  trace_stamp(a.trace, 21);

  // ---- 4: bulk copies of this CTA's share of each slot's expert: gate and up rows [FF*c/G, FF*(c+1)/G) on the slot's first
  // mbarrier, down rows [E*c/G, E*(c+1)/G) on its second; every gate/up request goes out before any down request ------------
  auto seg_src = [&](int k, int q) -> const uint8_t * {
    if (a.mode == 2 && a.slab[k]) {   // the store's copy: gate, up and down slabs back to back
      const uint8_t *b = a.slab[k];
      return q == 0 ? b + static_cast<size_t>(j0) * grb
           : q == 1 ? b + a.gate_slab + static_cast<size_t>(j0) * grb
                    : b + a.gate_slab + a.up_slab + static_cast<size_t>(i0) * drb;
    }
    const size_t e = static_cast<size_t>(s_spec[k]);
    return q == 0 ? a.gate + e * a.gate_slab + static_cast<size_t>(j0) * grb
         : q == 1 ? a.up + e * a.up_slab + static_cast<size_t>(j0) * grb
                  : a.down + e * a.down_slab + static_cast<size_t>(i0) * drb;
  };
  auto seg_off = [&](int k, int q) -> uint32_t {   // shared offset (from slots) of row 0 of segment q of slot k
    return static_cast<uint32_t>(k) * a.slot_bytes + (q == 0 ? 0u : q == 1 ? gseg : 2 * gseg) +
           static_cast<uint32_t>(reinterpret_cast<uintptr_t>(seg_src(k, q)) & 15u);
  };
  auto issue = [&](int k, bool down) {   // one thread: slot k's gate and up segments, or its down segment
    uint8_t *slot = slots + static_cast<size_t>(k) * a.slot_bytes;
    uint64_t *bar = down ? &dbar[k] : &bars[k];
    const int q0 = down ? 2 : 0, q1 = down ? 3 : 2;
    uint32_t total = 0;
    for (int q = q0; q < q1; ++q) {
      const uint32_t len = q < 2 ? static_cast<uint32_t>(ngu) * grb : static_cast<uint32_t>(nd) * drb;
      const uint32_t lo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(seg_src(k, q)) & 15u);
      total += len ? (lo + len + 15u) & ~15u : 0u;
    }
    mbar_arrive_expect_tx(bar, total);
    for (int q = q0; q < q1; ++q) {
      const uint32_t len = q < 2 ? static_cast<uint32_t>(ngu) * grb : static_cast<uint32_t>(nd) * drb;
      const uint8_t *src = seg_src(k, q);
      const uint32_t lo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src) & 15u);
      if (len) bulk_copy_g2s(slot + (q == 0 ? 0u : q == 1 ? gseg : 2 * gseg), src - lo, (lo + len + 15u) & ~15u, bar);
    }
  };
  if (my_rank < K) {   // the thread that ranked a chosen expert sends its gate and up rows at once
    issue(my_rank, false);
    s_iss[my_rank] = 1;
  }
  trace_stamp(a.trace, 23);
  __syncthreads();
  trace_stamp(a.trace, 11);
  const bool go = !s_flag[0] && a.mode != 1;
  // one thread per slot: the down rows after every gate/up request of the CTA, from warps that take no part in the softmax
  // where there are enough of them (an issue can wait while the copy unit takes the requests before it)
  const int k_iss = SW + K <= NW ? warp - SW : warp;
  if (go && k_iss >= 0 && k_iss < K && lane == 0) {
    const int k = k_iss;
    if (s_spec[k] < 0 || s_spec[k] >= NE || (spec && !(s_iss[k] & 1))) {   // logits that do not order (NaN)
      set_error(a.err, ERR_BAD_EXPERT);
      s_flag[0] = 1;
    } else {
      if (!spec) {
        issue(k, false);
        s_iss[k] = 1;
      }
      issue(k, true);
      s_iss[k] |= 2;
    }
  }
  trace_stamp(a.trace, 12);

  // ---- 3 (continued): softmax (double sum, c/src/forward.c:954-958), the probability order, the weights -----------------------
  if (a.mode != 2 && !s_flag[0]) {
    ev = tid < NE ? expf_cr(__fsub_rn(lv, mx)) : 0.f;
    double part = static_cast<double>(ev);   // each warp's 32 experts by a shuffle tree, then the warps in order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(FULL, part, o);
    if (lane == 0 && warp < SW) s_red[warp] = part;
  }
  __syncthreads();
  if (a.mode != 2 && !s_flag[0]) {
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < SW; ++w) tot += s_red[w];
    trace_stamp(a.trace, 9);
    if (tid < ((NE + 3) & ~3)) probs[tid] = tid < NE ? __double2float_rn(__ddiv_rn(static_cast<double>(ev), tot)) : -1.0f;
    trace_stamp(a.trace, 10);
  }
  __syncthreads();
  trace_stamp(a.trace, 20);
  bool need_rank = a.mode == 1;
  if (spec && !s_flag[0]) {
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
      if (lane == 0) s_flag[2] = strict ? 0 : 1;
    }
    __syncthreads();
    need_rank = s_flag[2] != 0;
  }
  if (need_rank && !s_flag[0]) {   // the full probability order
    const int e = tid >> 2;
    const int rank = rank4(probs, -1.0f);
    if (e < NE && (tid & 3) == 0 && rank < K) { s_sel[rank] = e; s_wt[rank] = probs[e]; }
  }
  __syncthreads();
  if (ahead && c == 0 && !s_flag[0]) {
    // router-ahead's choice (c/src/forward.c:940-945): repeated arg-max over the next layer's logits, ties to the lower
    // id, is the order of rank = experts with a larger logit + equal logits of lower ids
    if (tid < NE) lg2[tid] = __ldcg(a.logits + NE + tid);
    __syncthreads();
    if (tid < NE) {
      const float v = lg2[tid];
      int rank = 0;
#pragma unroll 4
      for (int f = 0; f < NE; ++f) {
        const float u = lg2[f];
        rank += (u > v) || (u == v && f < tid);
      }
      if (rank < a.ahead_n) a.ahead_out[rank] = tid;
    }
    __syncthreads();   // the slots are SMART-ROUTE's scratch next
  }
  if (a.mode == 1 && a.resident && c == 0 && !s_flag[0]) {
    // SMART-ROUTE (c/src/forward.c:961-969): cl_route's choice against the layer's resident set, each chosen expert weighted
    // by its own router probability; scratch in the expert slots, which routing-only launches leave unused
    double *rp = reinterpret_cast<double *>(slots);
    int *rorder = reinterpret_cast<int *>(rp + NE);
    uint8_t *rtaken = reinterpret_cast<uint8_t *>(rorder + NE);
    const SmartCfg cfg{1, a.smart_J, a.smart_M, a.smart_tau};
    route_cta(a.logits, NE, K, cfg, a.resident, rp, rorder, rtaken, s_red, s_sel, static_cast<RouteStats *>(a.smart_stats));
    if (tid < K) s_wt[tid] = probs[s_sel[tid]];
    __syncthreads();
  }
  if (spec && need_rank && !s_flag[0]) {
    // which slot holds each chosen expert; a slot holding an expert outside the top k takes a missing one (both in order)
    const int tk0 = tid < K ? s_sel[tid] : 0;
    if (warp == 0 && __any_sync(FULL, tk0 < 0 || tk0 >= NE)) {   // logits that do not order (NaN): no expert to fetch
      if (lane == 0) { set_error(a.err, ERR_BAD_EXPERT); s_flag[0] = 1; }
    } else if (warp == 0) {
      int gk = -1;
      const int tk = lane < K ? s_sel[lane] : -2;
      for (int h = 0; h < K; ++h) gk = s_spec[h] == tk ? h : gk;
      const int sg = lane < K ? s_spec[lane] : -2;
      bool in = false;
      for (int k = 0; k < K; ++k) in |= s_sel[k] == sg;
      const uint32_t orphan = __ballot_sync(FULL, lane < K && !in), missing = __ballot_sync(FULL, lane < K && gk < 0);
      if (lane < K && gk < 0) {   // the missing rank's position among the missing ranks pairs it with the orphan at the same position
        const int pos = __popc(missing & ((1u << lane) - 1u));
        uint32_t o = orphan;
        for (int t = 0; t < pos && o; ++t) o &= o - 1u;
        gk = o ? __ffs(o) - 1 : -1;
        if (gk >= 0) s_fix[gk] = tk + 1;
      }
      if (lane < K) s_slot[lane] = gk;
      if (lane < K && (gk < 0 || tk < 0)) { set_error(a.err, ERR_BAD_EXPERT); s_flag[0] = 1; }   // two sets of K: cannot happen
    }
    __syncthreads();
    if (warp < K && lane == 0 && s_fix[warp] && !s_flag[0]) {   // the wrong copies land first; then the right expert's
      const int k = warp;
      if (mbar_wait_bounded(&bars[k], 0) && mbar_wait_bounded(&dbar[k], 0)) {
        s_spec[k] = s_fix[k] - 1;
        issue(k, false);
        issue(k, true);
        s_par[k] = 1;
      } else {
        set_error(a.err, ERR_WAIT_COPY);
        s_flag[0] = 1;
      }
    }
    __syncthreads();
  }
  if (a.mode != 2 && !s_flag[0] && warp == 0) {   // renormalise: every lane forms the same sum in rank order, by shuffles
    const float wk = lane < K ? s_wt[lane] : 0.f;
    float z = 0.f;
#pragma unroll 8
    for (int k = 0; k < K; ++k) z = __fadd_rn(z, __shfl_sync(FULL, wk, k));
    if (lane < K) {
      const float w = a.norm_topk && z > 0.f ? __fdiv_rn(wk, z) : wk;
      s_wn[lane] = w;   // read after the next block barrier
      if (c == 0) {
        if (a.sel_out) a.sel_out[lane] = s_sel[lane];
        if (a.wt_out) a.wt_out[lane] = w;
      }
    }
    trace_stamp(a.trace, 22);
  }

  // ---- 5: gate and up rows: a group of lanes per (expert, row), one lane per block -------------------------------------------
  const bool run = go && !s_flag[0];   // read after the last block barrier: the same in every thread
  if (run) {
    const int GL = nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : nb <= 8 ? 8 : 16;   // lanes per group
    const int lg = lane & (GL - 1), gpw = 32 / GL, ngroups = NW * gpw, gid = warp * gpw + lane / GL;
    const int tasks = K * ngu, base = lane - lg;
    const bool has_blk = lg < nb;
    BlockAct act;
    if (has_blk) load_block_act(xq_qs, xq_d, xq_bs, lg, act);
    int waited = -1;
    for (int t0 = 0; t0 < tasks; t0 += ngroups) {   // the same trip count in every warp
      const int t = t0 + gid;
      const bool valid = t < tasks;
      const int k = valid ? t / ngu : 0, j = valid ? t - k * ngu : 0;
      float tg = 0.f, tu = 0.f;
      if (valid) {
        while (waited < k) {   // slots land in rank order; wait for each once
          ++waited;
          if (!mbar_wait_bounded(&bars[waited], static_cast<uint32_t>(s_par[waited]))) set_error(a.err, ERR_WAIT_COPY);
          if (waited == 0) trace_stamp(a.trace, 25);
        }
        if (has_blk) {
#pragma unroll 1
          for (int m = 0; m < 2; ++m) {   // one copy of the code
            const float t = kq_block(GT, slots + seg_off(k, m) + static_cast<uint32_t>(j) * grb, lg, act);
            if (m == 0) tg = t; else tu = t;
          }
        }
        if (t0 == 0) trace_stamp(a.trace, 26);
      }
      float sg = 0.f, su = 0.f;   // the row's block terms in block order
      for (int b = 0; b < nb; ++b) {
        sg = __fadd_rn(sg, __shfl_sync(FULL, tg, base + b));
        su = __fadd_rn(su, __shfl_sync(FULL, tu, base + b));
      }
      if (valid && lg == 0) __stcg(a.hg + static_cast<size_t>(k) * FF + j0 + j, silu_mul(sg, su));
    }
    trace_stamp(a.trace, 13);
    __syncthreads();
    if (tid == 0) red_release_add(&a.sync[1], 1u);   // release: the CTA's hg rows, ordered by bar.sync
  }
  trace_stamp(a.trace, 14);

  // ---- 6: every expert's hg, down rows, combine in rank order, residual ------------------------------------------------------
  if (run && tid == 0 && !wait_counter(&a.sync[1], static_cast<uint32_t>(G))) { set_error(a.err, ERR_WAIT_EXPERT); s_flag[0] = 1; }
  __syncthreads();
  trace_stamp(a.trace, 15);
  if (run && !s_flag[0]) {
    q8k_quantize_global(a.hg, K * FF / 256, hq_qs, hq_d, hq_bs, warp, NW, lane, true);
    trace_stamp(a.trace, 16);
    for (int k = 0; k < K; ++k)   // every copy has landed (a CTA with no gate/up rows has not waited yet)
      if (!mbar_wait_bounded(&dbar[k], static_cast<uint32_t>(s_par[k]))) set_error(a.err, ERR_WAIT_COPY);
    __syncthreads();
    trace_stamp(a.trace, 17);
    // (expert, block) pairs, LP lanes each, one row per lane: a pair's activation block is the same address for its lanes,
    // so its register copy costs one broadcast read per warp instead of one read per row
    const int C = K * nbd, LP = nd > 16 ? 32 : 16, ppw = 32 / LP, lp = lane & (LP - 1);
    for (int p = warp * ppw + lane / LP; p < C; p += NW * ppw) {
      const int k = p / nbd, blk = p - k * nbd;
      BlockAct dact;
      load_block_act(hq_qs, hq_d, hq_bs, p, dact);   // block index over all experts (k * nbd + blk): the swizzle key
      const uint8_t *drows = slots + seg_off(k, 2);
      for (int r = lp; r < nd; r += LP) terms[(r * K + k) * nbd + blk] = kq_block(DT, drows + static_cast<size_t>(r) * drb, blk, dact);
    }
    __syncthreads();
    trace_stamp(a.trace, 18);
    float *wprod = rprod;   // [nd][K] (the router products are done with)
    for (int q = tid; q < nd * K; q += DECODE_THREADS) {   // wt[k] * hd[r][k] for rank k, hd as the block terms in block order
      const int r = q / K, rk = q - r * K;
      const float *tq = terms + (r * K + s_slot[rk]) * nbd;   // the terms are by slot
      float hd = 0.f;
#pragma unroll 4
      for (int b = 0; b < nbd; ++b) hd = __fadd_rn(hd, tq[b]);
      wprod[q] = __fmul_rn(s_wn[q % K], hd);   // q = row * K + rank
    }
    __syncthreads();
    for (int r = tid; r < nd; r += DECODE_THREADS) {   // moe in rank order
      float moe = 0.f;
#pragma unroll 8
      for (int k = 0; k < K; ++k) moe = __fadd_rn(moe, wprod[r * K + k]);
      a.x_out[i0 + r] = __fadd_rn(xr[r], __fmul_rn(a.resid_scale, moe));
    }
  }

  // ---- exit: copies in flight land first; the last CTA out resets the counters ----------------------------------------------
  __syncthreads();
  trace_stamp(a.trace, 19);
  trace_time(a.trace, 31);
  if (tid == 0) {
    if (s_flag[0])   // an error path may leave copies unwaited; the normal path waited in phase 6
      for (int k = 0; k < K; ++k)
        if (((s_iss[k] & 1) && !mbar_wait_bounded(&bars[k], static_cast<uint32_t>(s_par[k]))) ||
            ((s_iss[k] & 2) && !mbar_wait_bounded(&dbar[k], static_cast<uint32_t>(s_par[k]))))
          set_error(a.err, ERR_WAIT_COPY);
    // a host call reads the results from host-mapped memory as soon as the error word arrives there: the CTA's writes
    // (x, sel and wt included, ordered by the block barrier) reach the host before its count
    if (a.err_out) __threadfence_system();
    const uint32_t prev = atomicAdd(&a.sync[2], 1u);
    if (prev == static_cast<uint32_t>(G) - 1) {
      if (a.err_out) {
        __threadfence_system();
        *reinterpret_cast<volatile int *>(a.err_out) = atomicOr(a.err, 0);
      }
      atomicExch(&a.sync[0], 0u);
      atomicExch(&a.sync[1], 0u);
      atomicExch(&a.sync[2], 0u);
      __threadfence();
    }
  }
}


__global__ void __launch_bounds__(256) stage_in_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst, int n4) {
  grid_launch_dependents();
  float4 v[4];
#pragma unroll
  for (int u = 0; u < 4; ++u)   // every load in flight before the first store: one round trip over the bus
    if (threadIdx.x + 256 * u < n4) v[u] = src[threadIdx.x + 256 * u];
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (threadIdx.x + 256 * u < n4) dst[threadIdx.x + 256 * u] = v[u];
}

cudaError_t launch_stage_in(const float *src, float *dst, int n, cudaStream_t st) {
  if (n % 4 || n > 4096) return cudaErrorInvalidValue;
  stage_in_kernel<<<1, 256, 0, st>>>(reinterpret_cast<const float4 *>(src), reinterpret_cast<float4 *>(dst), n / 4);
  return cudaGetLastError();
}

cudaError_t decode_allow_smem(int bytes) {
  const DecodeFn fns[4] = {moe_decode_kernel<T_Q4_K, T_Q4_K>, moe_decode_kernel<T_Q4_K, T_Q6_K>, moe_decode_kernel<T_Q6_K, T_Q4_K>,
                           moe_decode_kernel<T_Q6_K, T_Q6_K>};
  for (DecodeFn f : fns) {
    const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

DecodeFn decode_kernel_for(uint32_t gate_type, uint32_t down_type) {
  if (gate_type == T_Q4_K) return down_type == T_Q4_K ? moe_decode_kernel<T_Q4_K, T_Q4_K> : down_type == T_Q6_K ? moe_decode_kernel<T_Q4_K, T_Q6_K> : nullptr;
  if (gate_type == T_Q6_K) return down_type == T_Q4_K ? moe_decode_kernel<T_Q6_K, T_Q4_K> : down_type == T_Q6_K ? moe_decode_kernel<T_Q6_K, T_Q6_K> : nullptr;
  return nullptr;
}

}  // namespace clb
