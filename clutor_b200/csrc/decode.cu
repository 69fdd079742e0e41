// The one-token MoE block as one persistent kernel: the reference's c/src/forward.c:949-1033 on one B200.
//
// Modes (DecodeArgs::mode): 0 runs every phase below; 1 stops after phase 3 (routing only, for a host that must see the
// choice before it places the experts -- the expert store); 2 skips the router (phases 2-3) and takes the routing and the
// experts' addresses from its arguments (the experts as the store placed them in HBM).
//
// One CTA per SM (G CTAs, all co-resident), 512 threads. Every CTA streams the same share of every chosen expert, and all
// of a CTA's share of the chosen experts sits in shared memory at once. Data that crosses CTAs goes through global memory
// behind two counters (bounded waits):
//   0  (before the programmatic-launch wait, overlapping the previous kernel's tail) barriers; this CTA's router rows
//      (experts c, c+G, ...) and the norm weights start streaming into shared memory;
//   1  x, xn = rmsnorm(x) with a double sum of squares; the Q8_K blocks of xn;
//   2  router: all threads form the products router[e][i] * xn[i]; eight lanes per expert then add them as the reference's
//      dotf does -- eight strided float sums in element order, combined ((0+1)+(2+3))+((4+5)+(6+7)); logits to global
//      memory, counter 0 += experts scored;
//   3  when counter 0 reaches NE: softmax, top-k by rank counting (ties to the lower id, the order of the reference's
//      repeated arg-max), renormalisation; every CTA does this itself;
//   4  one lane per chosen expert issues the bulk copies of this CTA's share of it: gate and up rows [FF*c/G, FF*(c+1)/G),
//      down rows [E*c/G, E*(c+1)/G);
//   5  gate and up rows of all experts as they land, one lane per 256-element block (exact integer sums, the reference's
//      float block term), the terms of a row added in block order; SwiGLU; hg rows to global memory; counter 1 += 1;
//   6  when counter 1 reaches G: the Q8_K blocks of every expert's hg; down rows (same arithmetic); per output row
//      moe = sum over experts in rank order of wt * hd; x = x + resid_scale * moe; the last CTA out resets the counters.
#include "common.cuh"
#include "decode.cuh"
#include "rowdot.cuh"

namespace clb {

__global__ void __launch_bounds__(DECODE_THREADS, 1) moe_decode_kernel(const DecodeArgs a) {
  constexpr int NW = DECODE_THREADS / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int E = a.E, FF = a.FF, NE = a.NE, K = a.K;
  const int nb = E / 256, nbd = FF / 256;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bars);   // [K] expert slots, [K] router rows + norm weights
  float *xn = reinterpret_cast<float *>(smem + a.off_xn);             // [E] x, then xn
  float *wn = reinterpret_cast<float *>(smem + a.off_norm);           // [E] norm weights
  int8_t *xq_qs = reinterpret_cast<int8_t *>(smem + a.off_xq);        // Q8_K of xn: qs [E], bsums [E/16], d [E/256]
  int16_t *xq_bs = reinterpret_cast<int16_t *>(smem + a.off_xq + E);
  float *xq_d = reinterpret_cast<float *>(smem + a.off_xq + E + 2 * (E / 16));
  float *rrows = reinterpret_cast<float *>(smem + a.off_router);      // [nre][E] router rows, then their products
  double *s_red = reinterpret_cast<double *>(smem + a.off_misc);      // [NW]
  int *s_flag = reinterpret_cast<int *>(s_red + NW);                   // [0] failed, [1] copies issued
  int *s_sel = s_flag + 4;                                             // [32]
  float *s_wt = reinterpret_cast<float *>(s_sel + 32);                 // [32]
  float *s_mx = s_wt + 32;                                             // [NW]
  float *probs = s_mx + NW;                                            // [NE rounded up to 4]
  float *terms = reinterpret_cast<float *>(smem + a.off_terms);       // block terms of the rows of one phase
  float *gres = reinterpret_cast<float *>(smem + a.off_gres);         // [2 * K * rgu_max] gate/up row values
  uint32_t *rowoff = reinterpret_cast<uint32_t *>(smem + a.off_rowoff);   // [2 * K * rgu_max] shared offsets of gate/up rows
  int8_t *hq_qs = reinterpret_cast<int8_t *>(smem + a.off_hq);        // Q8_K of every expert's hg: qs [K*FF], bsums, d
  int16_t *hq_bs = reinterpret_cast<int16_t *>(smem + a.off_hq + K * FF);
  float *hq_d = reinterpret_cast<float *>(smem + a.off_hq + K * FF + 2 * (K * FF / 16));
  float *xr = reinterpret_cast<float *>(smem + a.off_xr);             // [rd_max] this CTA's rows of x
  float *hdv = reinterpret_cast<float *>(smem + a.off_hd);            // [rd_max * K] down row values per expert
  uint8_t *slots = smem + a.off_slots;

  const int j0 = static_cast<int>((static_cast<long long>(FF) * c) / G), j1 = static_cast<int>((static_cast<long long>(FF) * (c + 1)) / G);
  const int i0 = static_cast<int>((static_cast<long long>(E) * c) / G), i1 = static_cast<int>((static_cast<long long>(E) * (c + 1)) / G);
  const int ngu = j1 - j0, nd = i1 - i0;
  const int nre = (a.mode != 2 && c < NE) ? (NE - c + G - 1) / G : 0;   // experts this CTA scores: c, c+G, ...
  const uint32_t grb = a.grb, drb = a.drb, gseg = a.gseg;

  // ---- 0: barriers, router rows and norm weights (weights only, so before the dependency wait) ------------------------------
  if (tid == 0) {
    for (int s = 0; s <= K; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bars[K], static_cast<uint32_t>(nre + 1) * E * 4u);
    bulk_copy_g2s(wn, a.norm, E * 4u, &bars[K]);
    for (int m = 0; m < nre; ++m)
      bulk_copy_g2s(rrows + static_cast<size_t>(m) * E, a.router + static_cast<size_t>(c + m * G) * E, E * 4u, &bars[K]);
    s_flag[0] = 0;
    s_flag[1] = 0;
  }
  grid_dependency_wait();   // x, the scratch and the counters belong to the previous kernel until here
  grid_launch_dependents();

  // ---- 1: rmsnorm (double sum of squares; c/src/forward.c:412-417) and the Q8_K blocks of xn --------------------------------
  {
    double ss = 0.0;
    for (int i = tid * 4; i < E; i += DECODE_THREADS * 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x_in + i));
      reinterpret_cast<float4 *>(xn + i)[0] = v;
      ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
    if (lane == 0) s_red[warp] = ss;
    if (!mbar_wait_bounded(&bars[K], 0)) set_error(a.err, ERR_WAIT_COPY);
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += s_red[w];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / static_cast<double>(E)), a.eps)));
    for (int i = tid; i < nd; i += DECODE_THREADS) xr[i] = xn[i0 + i];
    __syncthreads();
    for (int i = tid; i < E; i += DECODE_THREADS) xn[i] = __fmul_rn(__fmul_rn(xn[i], scale), wn[i]);
    __syncthreads();
    // products of the router rows (in place) by every thread; the Q8_K blocks of xn wait until the copies are out
    for (int m = 0; m < nre; ++m)
      for (int i = tid; i < E; i += DECODE_THREADS) rrows[m * E + i] = __fmul_rn(rrows[m * E + i], xn[i]);
    __syncthreads();
  }

  // ---- 2: this CTA's router logits, the adds of the reference's dotf (c/src/forward.c:574-581) ---------------------------
  if (nre > 0) {
    const int grp = tid >> 3, l8 = tid & 7;
    if (warp * 4 < nre) {            // warp-uniform: a warp holds four 8-lane groups
      float s = 0.f;
      if (grp < nre) {
        const float *p = rrows + static_cast<size_t>(grp) * E + l8;
        for (int i = 0; i < E; i += 256) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = p[i + 8 * j];
#pragma unroll
          for (int j = 0; j < 32; ++j) s = __fadd_rn(s, v[j]);
        }
      }
      float p8[8];
#pragma unroll
      for (int l = 0; l < 8; ++l) p8[l] = __shfl_sync(FULL, s, (lane & ~7) + l);
      if (grp < nre && l8 == 0)
        a.logits[c + grp * G] = __fadd_rn(__fadd_rn(__fadd_rn(p8[0], p8[1]), __fadd_rn(p8[2], p8[3])),
                                          __fadd_rn(__fadd_rn(p8[4], p8[5]), __fadd_rn(p8[6], p8[7])));
    }
    __syncthreads();
    if (tid == 0) red_release_add(&a.sync[0], static_cast<uint32_t>(nre));   // release: the CTA's logits, ordered by bar.sync
  }

  // ---- 3: softmax, top-k, renormalisation (c/src/forward.c:954-984), in every CTA --------------------------------------------
  if (a.mode == 2) {   // the routing is given
    if (tid < K) {
      const int e = a.sel_in[tid];
      if (e < 0 || e >= NE) { set_error(a.err, ERR_BAD_EXPERT); s_flag[0] = 1; }
      s_sel[tid] = e;
      s_wt[tid] = a.wt_in[tid];
    }
  } else if (tid == 0 && !wait_counter(&a.sync[0], static_cast<uint32_t>(NE))) {
    set_error(a.err, ERR_WAIT_ROUTER);
    s_flag[0] = 1;
  }
  __syncthreads();
  if (a.mode != 2 && !s_flag[0]) {
    const float l = tid < NE ? __ldcg(a.logits + tid) : -INFINITY;
    float mx = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0) s_mx[warp] = mx;
    __syncthreads();
    mx = s_mx[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s_mx[w]);
    const float ev = tid < NE ? expf_cr(__fsub_rn(l, mx)) : 0.f;
    double sum = static_cast<double>(ev);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += s_red[w];
    const float p = __double2float_rn(__ddiv_rn(static_cast<double>(ev), tot));
    if (tid < ((NE + 3) & ~3)) probs[tid] = tid < NE ? p : -1.0f;
    __syncthreads();
    {   // rank = experts ahead of this one in the reference's arg-max order; four threads per expert, a quarter each
      const int e = tid >> 2, part = tid & 3, n4 = (NE + 3) / 4, per = (n4 + 3) / 4;
      const float pe = e < NE ? probs[e] : 0.f;
      int rank = 0;
      const float4 *p4 = reinterpret_cast<const float4 *>(probs);
      for (int j = part * per; j < min(n4, (part + 1) * per); ++j) {
        const float4 q = p4[j];
        const int f = 4 * j;
        rank += (q.x > pe || (q.x == pe && f < e)) + (q.y > pe || (q.y == pe && f + 1 < e)) +
                (q.z > pe || (q.z == pe && f + 2 < e)) + (q.w > pe || (q.w == pe && f + 3 < e));
      }
      rank += __shfl_xor_sync(FULL, rank, 1);
      rank += __shfl_xor_sync(FULL, rank, 2);
      if (e < NE && part == 0 && rank < K) { s_sel[rank] = e; s_wt[rank] = pe; }
    }
    __syncthreads();
    if (tid < K) {   // renormalise: each of K threads forms the same sum in rank order
      float w = s_wt[tid];
      if (a.norm_topk) {
        float z = 0.f;
        for (int k = 0; k < K; ++k) z = __fadd_rn(z, s_wt[k]);
        if (z > 0.f) w = __fdiv_rn(w, z);
      }
      __syncwarp(__activemask());
      s_wt[tid] = w;
      if (c == 0) {
        if (a.sel_out) a.sel_out[tid] = s_sel[tid];
        if (a.wt_out) a.wt_out[tid] = w;
      }
    }
  }
  __syncthreads();

  // ---- 4: bulk copies of this CTA's share of each chosen expert, one lane per expert ------------------------------------------
  auto seg_src = [&](int k, int q) -> const uint8_t * {
    if (a.mode == 2 && a.slab[k]) {   // the store's copy: gate, up and down slabs back to back
      const uint8_t *b = a.slab[k];
      return q == 0 ? b + static_cast<size_t>(j0) * grb
           : q == 1 ? b + a.gate_slab + static_cast<size_t>(j0) * grb
                    : b + a.gate_slab + a.up_slab + static_cast<size_t>(i0) * drb;
    }
    const size_t e = static_cast<size_t>(s_sel[k]);
    return q == 0 ? a.gate + e * a.gate_slab + static_cast<size_t>(j0) * grb
         : q == 1 ? a.up + e * a.up_slab + static_cast<size_t>(j0) * grb
                  : a.down + e * a.down_slab + static_cast<size_t>(i0) * drb;
  };
  auto seg_off = [&](int k, int q) -> uint32_t {   // shared offset (from slots) of row 0 of segment q of expert k
    return static_cast<uint32_t>(k) * a.slot_bytes + (q == 0 ? 0u : q == 1 ? gseg : 2 * gseg) +
           static_cast<uint32_t>(reinterpret_cast<uintptr_t>(seg_src(k, q)) & 15u);
  };
  const bool go = !s_flag[0] && a.mode != 1;
  if (go && lane == 0 && warp < K) {   // one warp per expert: their copy requests go out in parallel
    const int k = warp;
    uint8_t *slot = slots + static_cast<size_t>(k) * a.slot_bytes;
    const uint32_t len[3] = {static_cast<uint32_t>(ngu) * grb, static_cast<uint32_t>(ngu) * grb, static_cast<uint32_t>(nd) * drb};
    uint8_t *dst[3] = {slot, slot + gseg, slot + 2 * gseg};
    uint32_t total = 0, lo[3], n16[3];
    const uint8_t *src[3];
    for (int q = 0; q < 3; ++q) {
      src[q] = seg_src(k, q);
      lo[q] = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src[q]) & 15u);
      n16[q] = len[q] ? (lo[q] + len[q] + 15u) & ~15u : 0u;
      total += n16[q];
    }
    mbar_arrive_expect_tx(&bars[k], total);
    for (int q = 0; q < 3; ++q)
      if (n16[q]) bulk_copy_g2s(dst[q], src[q] - lo[q], n16[q], &bars[k]);
    if (k == 0) s_flag[1] = 1;
  }
  // while the copies fly: the Q8_K blocks of xn, and the offsets of the gate/up rows in task order (expert, gate/up, row)
  if (go) q8k_quantize_block(xn, E, xq_qs, xq_d, xq_bs, warp, NW, lane, true);
  const int per_k = 2 * ngu, tasks = K * per_k;
  if (go)
    for (int t = tid; t < tasks; t += DECODE_THREADS) {
      const int k = t / per_k, m = (t - k * per_k) / ngu, j = t - k * per_k - m * ngu;
      rowoff[t] = seg_off(k, m) + static_cast<uint32_t>(j) * grb;
    }
  __syncthreads();

  // ---- 5: gate and up rows, one lane per block; each lane's activation block stays in registers ------------------------------
  if (go) {
    const int slots_per_pass = DECODE_THREADS / nb, blk = tid % nb, rs = tid / nb;
    BlockAct act;
    load_block_act(xq_qs, xq_d, xq_bs, blk, act);
    int waited = -1;
    for (int t0 = 0; t0 < tasks; t0 += slots_per_pass) {
      const int t = t0 + rs;
      if (t < tasks) {
        const int k = t / per_k;
        while (waited < k) {   // slots land in rank order; wait for each once
          ++waited;
          if (!mbar_wait_bounded(&bars[waited], 0)) set_error(a.err, ERR_WAIT_COPY);
        }
        terms[t * nb + blk] = kq_block(a.gate_type, slots + rowoff[t], blk, act);
      }
    }
    __syncthreads();
    for (int t = tid; t < tasks; t += DECODE_THREADS) {   // a row's block terms in block order
      float s = 0.f;
      for (int b = 0; b < nb; ++b) s = __fadd_rn(s, terms[t * nb + b]);
      gres[t] = s;
    }
    __syncthreads();
    for (int t = tid; t < K * ngu; t += DECODE_THREADS) {
      const int k = t / ngu, j = t - k * ngu;
      __stcg(a.hg + static_cast<size_t>(k) * FF + j0 + j, silu_mul(gres[k * per_k + j], gres[k * per_k + ngu + j]));
    }
    __syncthreads();
    if (tid == 0) red_release_add(&a.sync[1], 1u);   // release: the CTA's hg rows, ordered by bar.sync
  }

  // ---- 6: every expert's hg, down rows, combine in rank order, residual ------------------------------------------------------
  if (go && tid == 0 && !wait_counter(&a.sync[1], static_cast<uint32_t>(G))) { set_error(a.err, ERR_WAIT_EXPERT); s_flag[0] = 1; }
  __syncthreads();
  if (go && !s_flag[0]) {
    q8k_quantize_global(a.hg, K * FF / 256, hq_qs, hq_d, hq_bs, warp, NW, lane, true);
    for (int k = 0; k < K; ++k)   // every copy has landed (a CTA with no gate/up rows has not waited yet)
      if (!mbar_wait_bounded(&bars[k], 0)) set_error(a.err, ERR_WAIT_COPY);
    __syncthreads();
    const int C = K * nbd;                       // (block, expert) combinations, expert fastest (different banks)
    const int combo = tid % C, grp = tid / C, ngrp = DECODE_THREADS / C;
    if (grp < ngrp) {
      const int blk = combo / K, k = combo - blk * K;
      BlockAct dact;
      load_block_act(hq_qs, hq_d, hq_bs, k * nbd + blk, dact);   // block index over all experts: the swizzle key
      const uint8_t *drows = slots + seg_off(k, 2);
      for (int r = grp; r < nd; r += ngrp) terms[(r * K + k) * nbd + blk] = kq_block(a.down_type, drows + static_cast<size_t>(r) * drb, blk, dact);
    }
    __syncthreads();
    for (int q = tid; q < nd * K; q += DECODE_THREADS) {   // hd[r][k]: the block terms in block order
      float hd = 0.f;
      for (int b = 0; b < nbd; ++b) hd = __fadd_rn(hd, terms[q * nbd + b]);
      hdv[q] = hd;
    }
    __syncthreads();
    for (int r = tid; r < nd; r += DECODE_THREADS) {
      float moe = 0.f;
      for (int k = 0; k < K; ++k) moe = __fadd_rn(moe, __fmul_rn(s_wt[k], hdv[r * K + k]));
      a.x_out[i0 + r] = __fadd_rn(xr[r], __fmul_rn(a.resid_scale, moe));
    }
  }

  // ---- exit: copies in flight land first; the last CTA out resets the counters ----------------------------------------------
  __syncthreads();
  if (tid == 0) {
    if (s_flag[1] && s_flag[0])   // an error path may leave copies unwaited; the normal path waited in phase 6
      for (int k = 0; k < K; ++k)
        if (!mbar_wait_bounded(&bars[k], 0)) set_error(a.err, ERR_WAIT_COPY);
    const uint32_t prev = atomicAdd(&a.sync[2], 1u);
    if (prev == static_cast<uint32_t>(G) - 1) {
      atomicExch(&a.sync[0], 0u);
      atomicExch(&a.sync[1], 0u);
      atomicExch(&a.sync[2], 0u);
      __threadfence();
    }
  }
}

}  // namespace clb
