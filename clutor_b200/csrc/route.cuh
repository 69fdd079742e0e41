// SMART-ROUTE on the device: the reference's cl_route (c/src/route.c:13-52) for one token, run by one CTA.
//
// Plain routing ranks the experts by their softmax probability in double (exp of logit - max, divided by the sum formed
// in expert order), best first, ties to the lower id, and takes the first K. SMART-ROUTE then keeps the true top-J; each
// other slot whose expert is not resident (in HBM) takes the best-ranked resident expert inside the top M that is not
// used yet, if its probability is within tau of the one it replaces (slots in rank order; a slot with no candidate keeps
// its expert). The residency is a byte per expert (non-zero: resident), read where the reference calls its callback.
//
// Arithmetic: the maximum, the exponentials, the sum (sequential, in expert order, as the reference's loop), the division
// and the differences against tau are the reference's double operations; CUDA's double exp is within one ulp of the C
// library's, so a ranking or a tau test can differ only when two probabilities, or a difference and tau, are within an ulp.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace clb {

constexpr int ROUTE_MAX_E = 1024;   // CL_MAX_E (c/src/route.h:12)
constexpr unsigned ROUTE_FULL = 0xffffffffu;
constexpr int ROUTE_MAX_K = 32;     // CL_MAX_K (c/src/route.h:11)

// SMART-ROUTE settings (cl_smart, c/src/route.h:14) and the counters of one routing (cl_route_result, route.h:16-22).
struct SmartCfg {
  int enabled, J, M;
  double tau;
};
struct RouteStats {
  int substituted, pad;
  double dropped_mass, max_delta;
};

// One CTA routes one token: every thread calls this. logits: [E] floats in global memory (read through L2). resident:
// [E] bytes or null (then plain routing, as the reference without a callback). Scratch in shared memory: p [E] doubles,
// order [E] ints, taken [E] bytes, red [blockDim / 32] doubles. Writes sel [K] (shared) and, from thread 0, *st. Returns
// after a block barrier, so sel and st are visible to every thread.
CLB_DEV void route_cta(const float *logits, int E, int K, const SmartCfg &cfg, const uint8_t *resident, double *p, int *order,
                       uint8_t *taken, double *red, int *sel, RouteStats *st) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  // the maximum as the reference forms it (route.c:17-18): the first logit, then every larger one; NaNs after the first
  // are passed over, a NaN first logit stays
  float m = -INFINITY;
  for (int i = 1 + tid; i < E; i += nt) {
    const float v = __ldcg(logits + i);
    if (v > m) m = v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(ROUTE_FULL, m, o));
  if (lane == 0) red[warp] = static_cast<double>(m);
  __syncthreads();
  double mx = static_cast<double>(__ldcg(logits));
  {
    double rest = red[0];
    for (int w = 1; w < nw; ++w) rest = fmax(rest, red[w]);
    if (!(mx != mx) && rest > mx) mx = rest;
  }
  for (int i = tid; i < E; i += nt) {
    p[i] = exp(static_cast<double>(__ldcg(logits + i)) - mx);
    order[i] = i;   // a valid index everywhere, whatever the ranking below writes
    taken[i] = 0;
  }
  __syncthreads();
  if (tid == 0) {   // the sum in expert order (route.c:19)
    double sum = 0.0;
    for (int i = 0; i < E; ++i) sum += p[i];
    red[0] = sum;
  }
  __syncthreads();
  const double sum = red[0];
  for (int i = tid; i < E; i += nt) p[i] = __ddiv_rn(p[i], sum);
  __syncthreads();
  // rank of each expert in the order of route.c:7-11 (probability descending, ties to the lower id)
  for (int i = tid; i < E; i += nt) {
    const double pi = p[i];
    int r = 0;
    for (int j = 0; j < E; ++j) {
      const double pj = p[j];
      r += (pj > pi) || (pj == pi && j < i);
    }
    order[r] = i;
  }
  __syncthreads();
  if (warp == 0) {
    if (lane < K) sel[lane] = order[lane];
    int subs = 0;
    double dropped = 0.0, maxd = 0.0;
    if (cfg.enabled && resident) {
      const int J = cfg.J < 0 ? 0 : cfg.J > K ? K : cfg.J;
      const int M = cfg.M < K ? K : cfg.M > E ? E : cfg.M;
      bool cold_here = false;
      if (lane < K) {   // route.c:31-34: the top-J and the resident ones are taken, the others are cold slots
        const int e = order[lane];
        if (lane < J || resident[e]) taken[e] = 1;
        else cold_here = true;
      }
      unsigned cold = __ballot_sync(ROUTE_FULL, cold_here);
      __syncwarp();
      while (cold) {   // route.c:35-51, the cold slots in rank order
        const int rank = __ffs(cold) - 1;
        cold &= cold - 1;
        const double pr = p[order[rank]];
        int pick = -1;
        for (int j0 = 0; j0 < M && pick < 0; j0 += 32) {   // the best-ranked candidate: the lowest j that qualifies
          const int j = j0 + lane;
          bool ok = false;
          if (j < M && j != rank) {
            const int e = order[j];
            ok = !taken[e] && resident[e] && !(pr - p[e] > cfg.tau);
          }
          const unsigned b = __ballot_sync(ROUTE_FULL, ok);
          if (b) pick = j0 + __ffs(b) - 1;
        }
        if (pick < 0) {
          if (lane == 0) taken[order[rank]] = 1;
        } else {
          const double d = pr - p[order[pick]];
          if (lane == 0) {
            taken[order[pick]] = 1;
            sel[rank] = order[pick];
          }
          ++subs;
          dropped += d;
          if (d > maxd) maxd = d;
        }
        __syncwarp();
      }
    }
    if (lane == 0 && st) {
      st->substituted = subs;
      st->pad = 0;
      st->dropped_mass = dropped;
      st->max_delta = maxd;
    }
  }
  __syncthreads();
}

}  // namespace clb
