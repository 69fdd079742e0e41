// The one-token MoE block as one persistent kernel: the reference's c/src/forward.c:949-1033 on one B200.
//
// One CTA per SM (G CTAs, all co-resident). Phases, with the data that crosses CTAs in global memory and bounded waits:
//   0  (before the programmatic-launch wait, so it overlaps the previous kernel's tail) barriers set up, and this CTA's
//      router rows (expert c, c+G, ...) start streaming into shared memory with a bulk copy;
//   1  every CTA reads x and forms xn = rmsnorm(x) (double sum of squares) and its Q8_K blocks (shared memory);
//   2  router: each expert's logit is the reference's dotf, eight strided float sums in element order combined
//      ((0+1)+(2+3))+((4+5)+(6+7)), computed by eight lanes; logits go to global memory and a counter;
//   3  every CTA waits for all logits and repeats softmax, top-k (ties to the lower id) and renormalisation itself;
//   4  one thread issues bulk copies of this CTA's share of every chosen expert, in rank order, into smem slots: gate and up
//      rows [FF*c/G, FF*(c+1)/G) and down rows [E*c/G, E*(c+1)/G) (all slots at once when they fit, else a ring);
//   5  per expert k: gate and up row dots (bit-exact, rowdot.cuh), SwiGLU, hg rows to global memory, ready[k] += 1;
//      then, one expert behind, down for expert k-1: wait ready[k-1] == G, quantize hg[k-1] to Q8_K (or keep floats for
//      Q8_0), down row dots, moe[i] += wt * hd[i] in rank order;
//   6  x[i] = x[i] + resid_scale * moe[i] for this CTA's rows; the last CTA out resets the counters.
#include "common.cuh"
#include "decode.cuh"
#include "rowdot.cuh"

namespace clb {

__global__ void __launch_bounds__(DECODE_THREADS, 1) moe_decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = DECODE_THREADS / 32;
  const int G = gridDim.x, c = blockIdx.x;
  const int E = a.E, FF = a.FF, NE = a.NE, K = a.K;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bars);   // [nslot] slot barriers, [nslot] router barrier
  float *xn = reinterpret_cast<float *>(smem + a.off_xn);
  int8_t *xq_qs = reinterpret_cast<int8_t *>(smem + a.off_xq);
  float *xq_d = reinterpret_cast<float *>(smem + a.off_xq + E);
  int16_t *xq_bs = reinterpret_cast<int16_t *>(smem + a.off_xq + E + 4 * (E / 256));
  float *rrows = reinterpret_cast<float *>(smem + a.off_router);
  double *s_red = reinterpret_cast<double *>(smem + a.off_misc);   // [NW]
  int *s_flag = reinterpret_cast<int *>(s_red + NW);                  // [0] error seen
  int *s_sel = s_flag + 4;                                            // [32]
  float *s_wt = reinterpret_cast<float *>(s_sel + 32);                // [32]
  float *probs = s_wt + 32;                                           // [NE]
  uint8_t *hq = smem + a.off_hq;                                 // down activations: Q8_K (qs, d, bsums) or fp32 hg
  float *gres = reinterpret_cast<float *>(smem + a.off_gres);   // [2 * rgu_max] gate then up row results
  float *moe = reinterpret_cast<float *>(smem + a.off_moe);     // [rd_max]
  float *xr = moe + a.rd_max;                                   // [rd_max] this CTA's x rows
  uint8_t *slots = smem + a.off_slots;

  const int j0 = static_cast<int>((static_cast<long long>(FF) * c) / G), j1 = static_cast<int>((static_cast<long long>(FF) * (c + 1)) / G);
  const int i0 = static_cast<int>((static_cast<long long>(E) * c) / G), i1 = static_cast<int>((static_cast<long long>(E) * (c + 1)) / G);
  const int ngu = j1 - j0, nd = i1 - i0;
  const int nre = (NE - c + G - 1) / G > 0 ? (NE - c + G - 1) / G : 0;   // experts this CTA scores: c, c+G, ...
  const uint32_t grb = a.grb, drb = a.drb;

  // ---- phase 0: barriers and the router rows (weights only: safe before the dependency wait) ----------------------------
  if (tid == 0) {
    for (int s = 0; s <= a.nslot; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    if (nre > 0) {
      mbar_arrive_expect_tx(&bars[a.nslot], static_cast<uint32_t>(nre) * E * 4u);
      for (int m = 0; m < nre; ++m)
        bulk_copy_g2s(rrows + static_cast<size_t>(m) * E, a.router + static_cast<size_t>(c + m * G) * E, E * 4u, &bars[a.nslot]);
    }
    s_flag[0] = 0;
  }
  for (int r = tid; r < a.rd_max; r += DECODE_THREADS) moe[r] = 0.f;

  grid_dependency_wait();   // x, the scratch and the counters belong to the previous kernel until here
  grid_launch_dependents();

  // ---- phase 1: x, rmsnorm (double sum of squares), Q8_K of xn ------------------------------------------------------------
  double ss = 0.0;
  for (int i = tid * 4; i < E; i += DECODE_THREADS * 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x_in + i));
    reinterpret_cast<float4 *>(xn + i)[0] = v;
    ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
  if (lane == 0) s_red[warp] = ss;
  __syncthreads();
  double tot = 0.0;
#pragma unroll
  for (int w = 0; w < NW; ++w) tot += s_red[w];
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / static_cast<double>(E)), a.eps)));
  for (int i = tid; i < nd; i += DECODE_THREADS) xr[i] = xn[i0 + i];
  __syncthreads();
  for (int i = tid; i < E; i += DECODE_THREADS) xn[i] = __fmul_rn(__fmul_rn(xn[i], scale), __ldg(a.norm + i));
  __syncthreads();
  q8k_quantize_block(xn, E, xq_qs, xq_d, xq_bs, warp, NW, lane);

  // ---- phase 2: this CTA's router logits, the reference's dotf ------------------------------------------------------------
  if (nre > 0) {
    if (!mbar_wait_bounded(&bars[a.nslot], 0)) set_error(a.err, ERR_WAIT_COPY);
    const int grp = tid >> 3, l8 = tid & 7;
    if (warp * 4 < nre) {            // warp-uniform: a warp holds four 8-lane groups
      float s = 0.f;
      if (grp < nre) {
        const float *w = rrows + static_cast<size_t>(grp) * E;
        for (int i = l8; i < E; i += 8) s = __fadd_rn(s, __fmul_rn(w[i], xn[i]));
      }
      float p[8];
#pragma unroll
      for (int l = 0; l < 8; ++l) p[l] = __shfl_sync(FULL, s, (lane & ~7) + l);
      if (grp < nre && l8 == 0) {
        const float t = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])), __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
        a.logits[c + grp * G] = t;
      }
    }
    __syncthreads();
    if (tid == 0) { __threadfence(); red_release_add(&a.sync[0], static_cast<uint32_t>(nre)); }
  }

  // ---- phase 3: all logits -> softmax, top-k, renormalise (every CTA, warp 0) ---------------------------------------------
  if (tid == 0 && !wait_counter(&a.sync[0], static_cast<uint32_t>(NE))) { set_error(a.err, ERR_WAIT_ROUTER); s_flag[0] = 1; }
  __syncthreads();
  const bool failed_router = s_flag[0] != 0;
  if (warp == 0 && !failed_router) {
    float v[DECODE_MAX_NE / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < DECODE_MAX_NE / 32; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < NE ? __ldcg(a.logits + e) : -INFINITY;
      mx = fmaxf(mx, v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < DECODE_MAX_NE / 32; ++j) {
      const int e = lane + 32 * j;
      if (e < NE) { v[j] = expf_cr(__fsub_rn(v[j], mx)); sum += static_cast<double>(v[j]); }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
    uint32_t used = 0;
#pragma unroll
    for (int j = 0; j < DECODE_MAX_NE / 32; ++j) {
      const int e = lane + 32 * j;
      if (e < NE) { v[j] = __double2float_rn(__ddiv_rn(static_cast<double>(v[j]), sum)); probs[e] = v[j]; }
      else used |= 1u << j;
    }
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
      if (c == 0) {
        for (int k = 0; k < K; ++k) {
          if (a.sel_out) a.sel_out[k] = s_sel[k];
          if (a.wt_out) a.wt_out[k] = s_wt[k];
        }
      }
    }
  }
  __syncthreads();

  // ---- phase 4: bulk copies of this CTA's share of each chosen expert ----------------------------------------------------
  const uint32_t gseg = a.gseg;   // bytes of the gate (= up) segment of a slot; the down segment follows both
  int last_issued = -1, last_consumed = -1;       // thread 0's record of the slot phases in flight
  auto issue = [&](int k) {                       // called by thread 0 only
    const int s = k % a.nslot;
    last_issued = k;
    uint8_t *slot = slots + static_cast<size_t>(s) * a.slot_bytes;
    const size_t e = static_cast<size_t>(s_sel[k]);
    const uint8_t *src[3] = {a.gate + e * a.gate_slab + static_cast<size_t>(j0) * grb, a.up + e * a.up_slab + static_cast<size_t>(j0) * grb,
                             a.down + e * a.down_slab + static_cast<size_t>(i0) * drb};
    const uint32_t len[3] = {static_cast<uint32_t>(ngu) * grb, static_cast<uint32_t>(ngu) * grb, static_cast<uint32_t>(nd) * drb};
    uint8_t *dst[3] = {slot, slot + gseg, slot + 2 * gseg};
    uint32_t total = 0, lo[3], n16[3];
    for (int q = 0; q < 3; ++q) {
      const uintptr_t p = reinterpret_cast<uintptr_t>(src[q]);
      lo[q] = static_cast<uint32_t>(p & 15u);
      n16[q] = len[q] ? (lo[q] + len[q] + 15u) & ~15u : 0u;
      total += n16[q];
    }
    fence_proxy_async();
    mbar_arrive_expect_tx(&bars[s], total);
    for (int q = 0; q < 3; ++q)
      if (n16[q]) bulk_copy_g2s(dst[q], src[q] - lo[q], n16[q], &bars[s]);
  };
  // where the rows of segment q start inside a slot (the copies start at the 16-byte boundary below the first row)
  auto seg_rows = [&](int k, int q) -> const uint8_t * {
    const size_t e = static_cast<size_t>(s_sel[k]);
    const uint8_t *src = q == 0 ? a.gate + e * a.gate_slab + static_cast<size_t>(j0) * grb
                         : q == 1 ? a.up + e * a.up_slab + static_cast<size_t>(j0) * grb
                                  : a.down + e * a.down_slab + static_cast<size_t>(i0) * drb;
    const uint8_t *slot = slots + static_cast<size_t>(k % a.nslot) * a.slot_bytes + (q == 0 ? 0 : q == 1 ? gseg : 2 * gseg);
    return slot + (reinterpret_cast<uintptr_t>(src) & 15u);
  };
  if (tid == 0 && !failed_router)
    for (int k = 0; k < K && k < a.nslot; ++k) issue(k);

  // activation registers for the gate/up rows (K-quants): the same xn for every expert
  const int nb_g = a.gate_type == T_Q8_0 ? E / 32 : E / 256;
  const RowShape rs_g = row_shape(a.gate_type == T_Q8_0 ? nb_g : 4 * nb_g);
  const int gsub = lane / rs_g.LG, glig = lane % rs_g.LG;
  KQAct act;
  if (a.gate_type != T_Q8_0) load_kq_act(a.gate_type, xq_qs, xq_d, xq_bs, nb_g, rs_g, glig, act);

  const int nb_d = a.down_type == T_Q8_0 ? FF / 32 : FF / 256;
  const RowShape rs_d = row_shape(a.down_type == T_Q8_0 ? nb_d : 4 * nb_d);
  const int dsub = lane / rs_d.LG, dlig = lane % rs_d.LG;
  float *hq_f = reinterpret_cast<float *>(hq);                         // [FF] hg of the expert being reduced
  int8_t *hq_qs = reinterpret_cast<int8_t *>(hq + 4 * FF);             // [FF] its Q8_K values
  float *hq_d = reinterpret_cast<float *>(hq + 5 * FF);                // [FF / 256]
  int16_t *hq_bs = reinterpret_cast<int16_t *>(hq + 5 * FF + 4 * (FF / 256));   // [FF / 16]

  auto gate_up = [&](int k) {
    const int s = k % a.nslot;
    if (!mbar_wait_bounded(&bars[s], static_cast<uint32_t>((k / a.nslot) & 1))) set_error(a.err, ERR_WAIT_COPY);
    last_consumed = k;
    const uint8_t *grow = seg_rows(k, 0), *urow = seg_rows(k, 1);
    const int tasks = 2 * ngu;
    for (int base = warp * rs_g.RPW; base < tasks; base += NW * rs_g.RPW) {
      const int task = base + gsub;
      const bool active = gsub < rs_g.RPW && task < tasks;
      const int r = task < ngu ? task : task - ngu;
      const uint8_t *row = (task < ngu ? grow : urow) + static_cast<size_t>(active ? r : 0) * grb;
      const float v = a.gate_type == T_Q8_0 ? q80_row(row, nb_g, rs_g, glig, gsub * rs_g.LG, xn, active)
                                            : kq_row(a.gate_type, row, nb_g, rs_g, glig, gsub * rs_g.LG, act, active);
      if (active && glig == 0) gres[task] = v;
    }
    __syncthreads();
    for (int r = tid; r < ngu; r += DECODE_THREADS) __stcg(a.hg + static_cast<size_t>(k) * FF + j0 + r, silu_mul(gres[r], gres[ngu + r]));
    __syncthreads();
    if (tid == 0) { __threadfence(); red_release_add(&a.sync[1 + k], 1u); }
  };

  auto down = [&](int k) {
    if (tid == 0 && !wait_counter(&a.sync[1 + k], static_cast<uint32_t>(G))) { set_error(a.err, ERR_WAIT_EXPERT); s_flag[0] = 1; }
    __syncthreads();
    if (s_flag[0]) return;
    for (int i = tid * 4; i < FF; i += DECODE_THREADS * 4)
      reinterpret_cast<float4 *>(hq_f)[i / 4] = __ldcg(reinterpret_cast<const float4 *>(a.hg + static_cast<size_t>(k) * FF + i));
    __syncthreads();
    KQAct dact;
    if (a.down_type != T_Q8_0) {
      q8k_quantize_block(hq_f, FF, hq_qs, hq_d, hq_bs, warp, NW, lane);
      __syncthreads();
      load_kq_act(a.down_type, hq_qs, hq_d, hq_bs, nb_d, rs_d, dlig, dact);
    }
    const uint8_t *drow = seg_rows(k, 2);
    const float w = s_wt[k];
    for (int base = warp * rs_d.RPW; base < nd; base += NW * rs_d.RPW) {
      const int r = base + dsub;
      const bool active = dsub < rs_d.RPW && r < nd;
      const uint8_t *row = drow + static_cast<size_t>(active ? r : 0) * drb;
      const float v = a.down_type == T_Q8_0 ? q80_row(row, nb_d, rs_d, dlig, dsub * rs_d.LG, hq_f, active)
                                            : kq_row(a.down_type, row, nb_d, rs_d, dlig, dsub * rs_d.LG, dact, active);
      if (active && dlig == 0) moe[r] = __fadd_rn(moe[r], __fmul_rn(w, v));
    }
    __syncthreads();
    if (tid == 0 && k + a.nslot < K) issue(k + a.nslot);
  };

  // ---- phase 5: experts in rank order, down one expert behind gate/up ------------------------------------------------------
  if (!failed_router) {
    for (int k = 0; k < K; ++k) {
      gate_up(k);
      if (k > 0) down(k - 1);
      if (s_flag[0]) break;
    }
    if (!s_flag[0]) down(K - 1);
  }

  // ---- phase 6: residual, then the last CTA resets the counters -----------------------------------------------------------
  __syncthreads();
  if (!s_flag[0])
    for (int r = tid; r < nd; r += DECODE_THREADS) a.x_out[i0 + r] = __fadd_rn(xr[r], __fmul_rn(a.resid_scale, moe[r]));
  if (tid == 0) {
    // copies issued but never consumed (an error path) must land before this CTA's shared memory is released
    for (int k = last_consumed + 1; k <= last_issued; ++k)
      if (!mbar_wait_bounded(&bars[k % a.nslot], static_cast<uint32_t>((k / a.nslot) & 1))) set_error(a.err, ERR_WAIT_COPY);
    __threadfence();
    const uint32_t prev = atomicAdd(&a.sync[K + 1], 1u);
    if (prev == static_cast<uint32_t>(G) - 1) {
      for (int q = 0; q <= K + 1; ++q) atomicExch(&a.sync[q], 0u);
      __threadfence();
    }
  }
}

}  // namespace clb
