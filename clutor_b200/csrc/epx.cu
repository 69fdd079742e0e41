// The exchange around the expert-parallel halves of the batched block (clb200_ep_route / clb200_ep_experts), on the device:
// the dispatch plan and the packed rows each token sends (one launch each), and the combine of the partial sums that come
// back (one launch). No counterpart in the reference, which runs on one machine; the arithmetic of the combine is the one
// the single-GPU block's combine does for a token's experts, with the experts grouped by rank (c/src/forward.c:1203-1208).
//
// Row format (the host driver's RowFormat): Q8_K qs [E] int8, d [E/256] fp32, bsums [E/16] int16, the token's expert ids
// made local to the destination [K] int32 (-1 where the expert is elsewhere), its weights [K] fp32; every part a multiple of
// 4 bytes, so rows are copied as 32-bit words.
#include "ctx.cuh"

using namespace clb;

namespace {

constexpr int EP_MAX_RANKS = 32;
constexpr int PLAN_THREADS = 1024;

// The destinations of token t: bit r set when rank r holds one of its experts (experts past the last rank go nowhere).
__device__ __forceinline__ uint32_t dest_mask(const int *sel, int t, int K, int n, int n_local) {
  uint32_t m = 0;
  for (int k = 0; k < K; ++k) {
    const int e = sel[static_cast<size_t>(t) * K + k];
    const int r = e >= 0 ? e / n_local : n;
    if (r < n) m |= 1u << r;
  }
  return m;
}

// One CTA: per rank the number of tokens it receives, and for every (token, rank) the row of the send buffer (ranks in
// order, tokens ascending within a rank) or -1.
__global__ void __launch_bounds__(PLAN_THREADS) ep_plan_kernel(const int *sel, int T, int K, int n, int n_local, int *slot, int *counts) {
  __shared__ int s_cnt[EP_MAX_RANKS], s_off[EP_MAX_RANKS], s_wsum[PLAN_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < EP_MAX_RANKS) s_cnt[tid] = 0;
  __syncthreads();
  for (int t = tid; t < T; t += PLAN_THREADS) {
    const uint32_t m = dest_mask(sel, t, K, n, n_local);
    for (int r = 0; r < n; ++r)
      if (m >> r & 1u) atomicAdd(&s_cnt[r], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0;
    for (int r = 0; r < n; ++r) {
      s_off[r] = o;
      o += s_cnt[r];
      counts[r] = s_cnt[r];
    }
  }
  __syncthreads();
  for (int base = 0; base < T; base += PLAN_THREADS) {   // tokens in order, a chunk at a time
    const int t = base + tid;
    const uint32_t m = t < T ? dest_mask(sel, t, K, n, n_local) : 0u;
    for (int r = 0; r < n; ++r) {
      const bool f = (m >> r & 1u) != 0;
      const uint32_t b = __ballot_sync(0xffffffffu, f);
      if (lane == 0) s_wsum[warp] = __popc(b);
      __syncthreads();
      int before = 0, total = 0;   // tokens of this chunk before this thread's warp, and in the whole chunk
      for (int w = 0; w < PLAN_THREADS / 32; ++w) {
        const int c = s_wsum[w];
        before += w < warp ? c : 0;
        total += c;
      }
      if (t < T) slot[static_cast<size_t>(t) * n + r] = f ? s_off[r] + before + __popc(b & ((1u << lane) - 1u)) : -1;
      __syncthreads();
      if (tid == 0) s_off[r] += total;
      __syncthreads();
    }
  }
}

// One CTA per token: its row for every rank it goes to.
__global__ void __launch_bounds__(128) ep_pack_kernel(const int *sel, const float *wt, const int8_t *qs, const float *d, const int16_t *bs,
                                                       int E, int K, int n, int n_local, const int *slot, uint8_t *send, int row_words) {
  const int t = blockIdx.x, tid = threadIdx.x;
  const int wq = E / 4, wd = E / 256, wb = E / 32;   // words of qs, d and bsums
  const uint32_t *sq = reinterpret_cast<const uint32_t *>(qs + static_cast<size_t>(t) * E);
  const uint32_t *sd = reinterpret_cast<const uint32_t *>(d + static_cast<size_t>(t) * (E / 256));
  const uint32_t *sb = reinterpret_cast<const uint32_t *>(bs + static_cast<size_t>(t) * (E / 16));
  for (int r = 0; r < n; ++r) {
    const int row = slot[static_cast<size_t>(t) * n + r];
    if (row < 0) continue;   // uniform over the CTA
    uint32_t *dst = reinterpret_cast<uint32_t *>(send) + static_cast<size_t>(row) * row_words;
    for (int i = tid; i < wq; i += 128) dst[i] = sq[i];
    for (int i = tid; i < wd; i += 128) dst[wq + i] = sd[i];
    for (int i = tid; i < wb; i += 128) dst[wq + wd + i] = sb[i];
    if (tid < K) {
      const int e = sel[static_cast<size_t>(t) * K + tid];
      const bool here = e >= 0 && e / n_local == r;
      dst[wq + wd + wb + tid] = static_cast<uint32_t>(here ? e - r * n_local : -1);
      dst[wq + wd + wb + K + tid] = __float_as_uint(wt[static_cast<size_t>(t) * K + tid]);
    }
  }
}

// One CTA per token: x += resid_scale * (its partial sums in rank order).
__global__ void __launch_bounds__(256) ep_combine_kernel(const int *slot, const float *back, float *x, int E, int n, float resid_scale) {
  const int t = blockIdx.x;
  int rows[EP_MAX_RANKS];
  int nr = 0;
  for (int r = 0; r < n; ++r) {
    const int s = slot[static_cast<size_t>(t) * n + r];
    if (s >= 0) rows[nr++] = s;
  }
  float *xr = x + static_cast<size_t>(t) * E;
  for (int i = threadIdx.x; i < E; i += 256) {
    float acc = 0.f;
    for (int j = 0; j < nr; ++j) acc = __fadd_rn(acc, back[static_cast<size_t>(rows[j]) * E + i]);
    xr[i] = __fadd_rn(xr[i], __fmul_rn(resid_scale, acc));
  }
}

bool ep_shape_ok(int T, int E, int K, int n, int n_local, char *err, size_t errlen) {
  if (T < 0 || E < 256 || E % 256 || K < 1 || K > DECODE_MAX_K || n < 1 || n > EP_MAX_RANKS || n_local < 1) {
    errf(err, errlen, "exchange of %d tokens, width %d, %d used over %d ranks of %d experts: out of range", T, E, K, n, n_local);
    return false;
  }
  return true;
}

}  // namespace

extern "C" {

int clb200_ep_pack(clb200_ctx *c, int T, int E, int K, int n_ranks, int n_local, const int *sel, const float *wt, const int8_t *xq_qs,
                   const float *xq_d, const int16_t *xq_bs, uint8_t *send, int *slot, int *counts, void *stream, char *err,
                   size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (!ep_shape_ok(T, E, K, n_ranks, n_local, err, errlen)) return 1;
  if (T == 0) return 0;
  if (!sel || !wt || !xq_qs || !xq_d || !xq_bs || !send || !slot || !counts) { errf(err, errlen, "a buffer is missing"); return 1; }
  cudaSetDevice(c->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  ep_plan_kernel<<<1, PLAN_THREADS, 0, st>>>(sel, T, K, n_ranks, n_local, slot, counts);
  const int row_words = (E + E / 64 + E / 8 + 8 * K) / 4;
  ep_pack_kernel<<<T, 128, 0, st>>>(sel, wt, xq_qs, xq_d, xq_bs, E, K, n_ranks, n_local, slot, send, row_words);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { errf(err, errlen, "launching the exchange packing: %s", cudaGetErrorString(e)); return 1; }
  return 0;
}

int clb200_ep_combine(clb200_ctx *c, int T, int E, int n_ranks, const int *slot, const float *back, float *x, float resid_scale,
                      void *stream, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (!ep_shape_ok(T, E, 1, n_ranks, 1, err, errlen)) return 1;
  if (T == 0) return 0;
  if (!slot || !back || !x) { errf(err, errlen, "a buffer is missing"); return 1; }
  cudaSetDevice(c->device);
  ep_combine_kernel<<<T, 256, 0, stream ? static_cast<cudaStream_t>(stream) : c->stream>>>(slot, back, x, E, n_ranks, resid_scale);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { errf(err, errlen, "launching the exchange combine: %s", cudaGetErrorString(e)); return 1; }
  return 0;
}

}  // extern "C"
