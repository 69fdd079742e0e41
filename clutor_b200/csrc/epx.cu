// The exchange around the expert-parallel halves of the batched block (clb200_ep_route / clb200_ep_experts), on the device:
// the dispatch plan and the packed rows each token sends (one launch each), and the combine of the partial sums that come
// back (one launch). No counterpart in the reference, which runs on one machine; the arithmetic of the combine is the one
// the single-GPU block's combine does for a token's experts, with the experts grouped by rank (c/src/forward.c:1203-1208).
//
// Row format (the host driver's RowFormat): Q8_K qs [E] int8, d [E/256] fp32, bsums [E/16] int16, the token's expert ids
// made local to the destination [K] int32 (-1 where the expert is elsewhere), its weights [K] fp32; every part a multiple of
// 4 bytes, so rows are copied as 32-bit words.
#include <cstring>

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

// ---- the exchange over peer memory (NVLink / NVSwitch), no library collective -----------------------------------------------
// Every rank allocates one exchange buffer of the same layout and maps every other rank's (CUDA IPC), so a kernel on one
// GPU stores straight into another GPU's memory. A rank's buffer:
//   [0, 4096)  header: 64-bit words [s] (rows from sender s: (sequence << 32) | rows) and [EP_MAX_RANKS + s] (partial
//              sums back from rank s: sequence << 32), written by the peers; two 32-bit launch counters at byte 1024
//              (this rank's own, for its push kernels' last-CTA release)
//   recv       [n][t_max] rows of row_bytes: region s holds the rows sender s dispatched here, tokens ascending
//   back       [n][t_max][E] fp32: region r holds the partial sums rank r returned for the rows sent to r, same order
// A kernel pushes every row with plain stores, each CTA fences at system scope and counts itself out; the last CTA out
// releases the (sequence, rows) word into each receiver's header. Receivers wait (bounded) on those words. A sender only
// overwrites a receiver's region after it has that receiver's partial sums of the previous step (the receiver returns them
// after its experts read the rows), so one buffer per rank suffices.
constexpr size_t XB_HDR = 4096, XB_CTR = 1024;
size_t xb_recv_bytes(int n, int t_max, int row_bytes) { return (static_cast<size_t>(n) * t_max * row_bytes + 255) & ~size_t(255); }
size_t xb_bytes(int n, int t_max, int row_bytes, int E) { return XB_HDR + xb_recv_bytes(n, t_max, row_bytes) + static_cast<size_t>(n) * t_max * E * 4; }

struct EpPeers {
  uint8_t *base[EP_MAX_RANKS];   // every rank's exchange buffer as this GPU addresses it (its own included)
};

__device__ __forceinline__ void st_release_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Copies `bytes` (a multiple of 4) from src to dst with the CTA's threads, 16 bytes at a time where both are aligned.
__device__ __forceinline__ void cta_copy(uint8_t *dst, const uint8_t *src, int bytes) {
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | static_cast<uintptr_t>(bytes)) & 15) == 0) {
    const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
    uint4 *d4 = reinterpret_cast<uint4 *>(dst);
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d4[i] = __ldcg(s4 + i);
  } else {
    const uint32_t *s1 = reinterpret_cast<const uint32_t *>(src);
    uint32_t *d1 = reinterpret_cast<uint32_t *>(dst);
    for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x) d1[i] = __ldcg(s1 + i);
  }
}

// Rows [0, S) of a list made of n regions (region r: cnt[r] rows): the region of row g and its index in the region.
__device__ __forceinline__ int region_of(const int *cnt, int n, int g, int *in) {
  int o = 0;
  for (int r = 0; r < n; ++r) {
    if (g < o + cnt[r]) { *in = g - o; return r; }
    o += cnt[r];
  }
  *in = 0;
  return -1;
}

// The last CTA out releases word (seq << 32) | rows[r] into header slot `slot` of every rank r: every thread fences its
// stores at system scope before its CTA counts itself out, and the last CTA fences again after seeing the count complete.
__device__ __forceinline__ void release_to_peers(const EpPeers &p, int n, int slot, uint32_t seq, const int *rows,
                                                 unsigned int *ctr) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int r = 0; r < n; ++r)
        st_release_sys_u64(reinterpret_cast<unsigned long long *>(p.base[r]) + slot,
                           (static_cast<unsigned long long>(seq) << 32) | static_cast<uint32_t>(rows ? rows[r] : 0));
      atomicExch(ctr, 0u);
    }
  }
}

// Pushes the send buffer's rows (regions by destination, counts[r] rows for rank r) into region `me` of each destination's
// receive area, then signals each destination with its row count.
__global__ void __launch_bounds__(256) ep_push_rows_kernel(const uint8_t *send, int row_bytes, const int *counts, int me, int n,
                                                           EpPeers p, int t_max, uint32_t seq, unsigned int *ctr) {
  __shared__ int s_cnt[EP_MAX_RANKS];
  if (threadIdx.x < n) s_cnt[threadIdx.x] = counts[threadIdx.x];
  __syncthreads();
  int S = 0;
  for (int r = 0; r < n; ++r) S += s_cnt[r];
  for (int g = blockIdx.x; g < S; g += gridDim.x) {
    int j;
    const int r = region_of(s_cnt, n, g, &j);
    if (r < 0 || j >= t_max) continue;   // cannot happen: counts come from the plan of at most t_max tokens
    cta_copy(p.base[r] + XB_HDR + (static_cast<size_t>(me) * t_max + j) * row_bytes, send + static_cast<size_t>(g) * row_bytes, row_bytes);
  }
  release_to_peers(p, n, me, seq, s_cnt, ctr);
}

// Pushes the partial sums of the rows each sender s dispatched here (rows [0, rcounts[s]) of region s of `partial`) back
// into region `me` of that sender's back area, then signals each sender.
__global__ void __launch_bounds__(256) ep_push_back_kernel(const float *partial, int E, const int *rcounts, int me, int n, EpPeers p,
                                                           int t_max, size_t recv_bytes, uint32_t seq, unsigned int *ctr) {
  __shared__ int s_cnt[EP_MAX_RANKS];
  if (threadIdx.x < n) s_cnt[threadIdx.x] = min(max(rcounts[threadIdx.x], 0), t_max);
  __syncthreads();
  int S = 0;
  for (int r = 0; r < n; ++r) S += s_cnt[r];
  for (int g = blockIdx.x; g < S; g += gridDim.x) {
    int j;
    const int s = region_of(s_cnt, n, g, &j);
    if (s < 0) continue;
    float *dst = reinterpret_cast<float *>(p.base[s] + XB_HDR + recv_bytes) + (static_cast<size_t>(me) * t_max + j) * E;
    cta_copy(reinterpret_cast<uint8_t *>(dst), reinterpret_cast<const uint8_t *>(partial + (static_cast<size_t>(s) * t_max + j) * E), E * 4);
  }
  release_to_peers(p, n, EP_MAX_RANKS + me, seq, nullptr, ctr);
}

// Waits (bounded) until header slots [slot0, slot0 + n) of this rank's buffer carry `seq`; their row counts to counts_out
// (when given). A slot that does not arrive sets the device error word and counts as 0 rows.
__global__ void __launch_bounds__(32) ep_wait_kernel(const unsigned long long *hdr, int slot0, int n, uint32_t seq, int *counts_out,
                                                     int *err) {
  const int s = threadIdx.x;
  if (s >= n) return;
  unsigned long long w = 0;
  bool got = false;
#pragma unroll 1
  for (uint32_t i = 0; i < SPIN_LIMIT; ++i) {
    w = ld_acquire_sys_u64(hdr + slot0 + s);
    if (static_cast<uint32_t>(w >> 32) == seq) { got = true; break; }
    if (i > 4096) __nanosleep(128);
  }
  if (!got) set_error(err, ERR_WAIT_PEER);
  if (counts_out) counts_out[s] = got ? static_cast<int>(static_cast<uint32_t>(w)) : 0;
}

// One CTA per token: x += resid_scale * (its partial sums in rank order), the partial sums from the back area: the row
// for rank r sits at r * t_max + (slot - the rows of the ranks before r).
__global__ void __launch_bounds__(256) ep_combine_regions_kernel(const int *slot, const int *counts, const float *back, float *x, int E,
                                                                 int n, int t_max, float resid_scale) {
  const int t = blockIdx.x;
  size_t rows[EP_MAX_RANKS];
  int nr = 0, off = 0;
  for (int r = 0; r < n; ++r) {
    const int s = slot[static_cast<size_t>(t) * n + r];
    if (s >= 0) rows[nr++] = static_cast<size_t>(r) * t_max + (s - off);
    off += counts[r];
  }
  float *xr = x + static_cast<size_t>(t) * E;
  for (int i = threadIdx.x; i < E; i += 256) {
    float acc = 0.f;
    for (int j = 0; j < nr; ++j) acc = __fadd_rn(acc, back[rows[j] * E + i]);
    xr[i] = __fadd_rn(xr[i], __fmul_rn(resid_scale, acc));
  }
}

int ep_row_bytes(int E, int K) { return E + E / 64 + E / 8 + 8 * K; }

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

void clb200_ep_xbuf_layout(int n_ranks, int t_max, int E, int n_used, size_t *bytes, size_t *recv_off, size_t *back_off) {
  const int rb = ep_row_bytes(E, n_used);
  if (bytes) *bytes = xb_bytes(n_ranks, t_max, rb, E);
  if (recv_off) *recv_off = XB_HDR;
  if (back_off) *back_off = XB_HDR + xb_recv_bytes(n_ranks, t_max, rb);
}

int clb200_ep_xbuf_alloc(clb200_ctx *c, int n_ranks, int t_max, int E, int n_used, void **buf, void *ipc_handle, char *err,
                         size_t errlen) {
  if (!c || !buf || !ipc_handle) { errf(err, errlen, "no context, buffer or handle"); return 1; }
  if (!ep_shape_ok(t_max, E, n_used, n_ranks, 1, err, errlen) || t_max < 1) {
    if (t_max < 1) errf(err, errlen, "an exchange buffer for %d tokens", t_max);
    return 1;
  }
  cudaSetDevice(c->device);
  const size_t bytes = xb_bytes(n_ranks, t_max, ep_row_bytes(E, n_used), E);
  *buf = nullptr;
  CUDA_OR(cudaMalloc(buf, bytes), "allocating the exchange buffer");
  CUDA_OR(cudaMemset(*buf, 0, bytes), "clearing the exchange buffer");
  CUDA_OR(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), *buf), "exporting the exchange buffer");
  return 0;
}

int clb200_ep_xbuf_open(clb200_ctx *c, const void *ipc_handle, void **peer, char *err, size_t errlen) {
  if (!c || !ipc_handle || !peer) { errf(err, errlen, "no context, handle or pointer"); return 1; }
  cudaSetDevice(c->device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof h);
  *peer = nullptr;
  CUDA_OR(cudaIpcOpenMemHandle(peer, h, cudaIpcMemLazyEnablePeerAccess), "mapping another rank's exchange buffer");
  return 0;
}

int clb200_ep_xbuf_close(clb200_ctx *c, void *peer, char *err, size_t errlen) {
  if (!c || !peer) { errf(err, errlen, "no context or pointer"); return 1; }
  cudaSetDevice(c->device);
  CUDA_OR(cudaIpcCloseMemHandle(peer), "unmapping another rank's exchange buffer");
  return 0;
}

int clb200_ep_xbuf_free(clb200_ctx *c, void *buf, char *err, size_t errlen) {
  if (!c || !buf) { errf(err, errlen, "no context or buffer"); return 1; }
  cudaSetDevice(c->device);
  CUDA_OR(cudaFree(buf), "freeing the exchange buffer");
  return 0;
}

static bool peers_of(void *const *bufs, int n, EpPeers &p, char *err, size_t errlen) {
  if (!bufs) { errf(err, errlen, "no exchange buffers"); return false; }
  for (int r = 0; r < n; ++r) {
    if (!bufs[r]) { errf(err, errlen, "rank %d's exchange buffer is not mapped", r); return false; }
    p.base[r] = static_cast<uint8_t *>(bufs[r]);
  }
  return true;
}

int clb200_ep_push(clb200_ctx *c, int me, int n_ranks, int t_max, int E, int n_used, void *const *bufs, const uint8_t *send,
                   const int *counts, unsigned int seq, void *stream, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (!ep_shape_ok(t_max, E, n_used, n_ranks, 1, err, errlen)) return 1;
  if (me < 0 || me >= n_ranks || !send || !counts) { errf(err, errlen, "rank %d of %d, or a buffer is missing", me, n_ranks); return 1; }
  EpPeers p{};
  if (!peers_of(bufs, n_ranks, p, err, errlen)) return 1;
  cudaSetDevice(c->device);
  unsigned int *ctr = reinterpret_cast<unsigned int *>(p.base[me] + XB_CTR);
  ep_push_rows_kernel<<<2 * c->sms, 256, 0, stream ? static_cast<cudaStream_t>(stream) : c->stream>>>(
      send, ep_row_bytes(E, n_used), counts, me, n_ranks, p, t_max, seq, ctr);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { errf(err, errlen, "launching the row push: %s", cudaGetErrorString(e)); return 1; }
  return 0;
}

int clb200_ep_wait(clb200_ctx *c, const void *own_buf, int n_ranks, int which, unsigned int seq, int *counts_out, void *stream,
                   char *err, size_t errlen) {
  if (!c || !own_buf) { errf(err, errlen, "no context or buffer"); return 1; }
  if (n_ranks < 1 || n_ranks > EP_MAX_RANKS || (which != 0 && which != 1)) { errf(err, errlen, "%d ranks, wait %d", n_ranks, which); return 1; }
  cudaSetDevice(c->device);
  ep_wait_kernel<<<1, 32, 0, stream ? static_cast<cudaStream_t>(stream) : c->stream>>>(
      static_cast<const unsigned long long *>(own_buf), which ? EP_MAX_RANKS : 0, n_ranks, seq, counts_out, c->small);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { errf(err, errlen, "launching the exchange wait: %s", cudaGetErrorString(e)); return 1; }
  return 0;
}

int clb200_ep_push_back(clb200_ctx *c, int me, int n_ranks, int t_max, int E, int n_used, void *const *bufs, const float *partial,
                        const int *rcounts, unsigned int seq, void *stream, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (!ep_shape_ok(t_max, E, n_used, n_ranks, 1, err, errlen)) return 1;
  if (me < 0 || me >= n_ranks || !partial || !rcounts) { errf(err, errlen, "rank %d of %d, or a buffer is missing", me, n_ranks); return 1; }
  EpPeers p{};
  if (!peers_of(bufs, n_ranks, p, err, errlen)) return 1;
  cudaSetDevice(c->device);
  unsigned int *ctr = reinterpret_cast<unsigned int *>(p.base[me] + XB_CTR) + 1;
  ep_push_back_kernel<<<2 * c->sms, 256, 0, stream ? static_cast<cudaStream_t>(stream) : c->stream>>>(
      partial, E, rcounts, me, n_ranks, p, t_max, xb_recv_bytes(n_ranks, t_max, ep_row_bytes(E, n_used)), seq, ctr);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { errf(err, errlen, "launching the partial-sum push: %s", cudaGetErrorString(e)); return 1; }
  return 0;
}

int clb200_ep_combine_regions(clb200_ctx *c, int T, int E, int n_ranks, int t_max, const int *slot, const int *counts,
                              const float *back, float *x, float resid_scale, void *stream, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (!ep_shape_ok(T, E, 1, n_ranks, 1, err, errlen) || T > t_max) {
    if (T > t_max) errf(err, errlen, "%d tokens, the exchange holds %d", T, t_max);
    return 1;
  }
  if (T == 0) return 0;
  if (!slot || !counts || !back || !x) { errf(err, errlen, "a buffer is missing"); return 1; }
  cudaSetDevice(c->device);
  ep_combine_regions_kernel<<<T, 256, 0, stream ? static_cast<cudaStream_t>(stream) : c->stream>>>(slot, counts, back, x, E, n_ranks,
                                                                                                   t_max, resid_scale);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { errf(err, errlen, "launching the exchange combine: %s", cudaGetErrorString(e)); return 1; }
  return 0;
}

}  // extern "C"
