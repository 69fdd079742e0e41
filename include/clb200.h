/*
 * clutor-b200: the Clutor engine's mixture-of-experts feed-forward block on NVIDIA B200 (sm_100a), behind a plain C ABI.
 *
 * Two ways in, both drop-ins for the reference engine's C host code:
 *
 *  1. clb200_moe_ffn(): the whole per-layer MoE block in one call. It replaces the inline block of the reference's forward
 *     pass, c/src/forward.c:949-1033 (one token: rmsnorm, router, softmax/top-k/renorm, Q8_K quantization, gate/up products,
 *     SwiGLU, down products, weighted combine, residual) and c/src/forward.c:1132-1210 (a batch of tokens: the same per token,
 *     with each chosen expert's weights read once for all the tokens that chose it). The layer description mirrors the
 *     fields the reference binds in cl_fwd_open (c/src/forward.h:18-29, c/src/forward.c:204-240).
 *
 *  2. clb200_backend(): a cl_backend (c/src/backend.h:9-13) named "b200" for the reference's plugin seam, cl_matvec_batch
 *     (c/src/quant.c:995-1004). Register it with cl_backend_register() and select it with CLUTOR_BACKEND=b200; it runs the
 *     Q4_K, Q6_K and Q8_0 products on the GPU and leaves every other type to the CPU, as the seam prescribes.
 *
 * Conventions follow the reference: functions that can fail return 0 on success and 1 on failure with a message written to
 * err (snprintf into errlen bytes), as cl_fwd_open / cl_fwd_step do (c/src/forward.c:24-27). No entry point falls back to
 * the CPU: without a usable CUDA device, clb200_open fails.
 *
 * Weights stay in their GGUF block layout on the device: the device format is the file format.
 */
#ifndef CLB200_H
#define CLB200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CLB200_ABI_VERSION 1

/* ggml tensor type ids, the values of the reference's CL_T_* (c/src/quant.h:7). Expert weights may be Q4_K, Q6_K or Q8_0. */
enum { CLB200_T_F32 = 0, CLB200_T_F16 = 1, CLB200_T_Q8_0 = 8, CLB200_T_Q4_K = 12, CLB200_T_Q6_K = 14 };

/* rows x cols weights of `type`, row-major, cols is the input width: the reference's cl_w (c/src/forward.h:18), same layout. */
typedef struct { const uint8_t *p; uint32_t type; int rows, cols; } clb200_w;

/* One MoE layer: what the reference's MoE block reads from cl_fwd_layer and cl_fwd (c/src/forward.h:20-29, 35-51).
 * gate/up/down are the fused expert tensors ffn_gate_exps / ffn_up_exps / ffn_down_exps: rows x cols is ONE expert
 * (gate/up: n_ff_exp x n_embd, down: n_embd x n_ff_exp) and n_expert slabs of gate_slab / up_slab / down_slab bytes follow
 * one another. ffn_norm_f and router_f are the fp32 copies the reference makes at load time (c/src/forward.c:234-239). */
typedef struct {
  const float *ffn_norm_f;   /* [n_embd] */
  const float *router_f;     /* [n_expert * n_embd], row e scores expert e */
  clb200_w gate, up, down;
  uint64_t gate_slab, up_slab, down_slab;
  int n_embd, n_ff_exp, n_expert, n_used;
  int norm_topk;             /* 1: renormalise the chosen weights to sum to 1 (qwen3moe, granitemoe); 0: raw probabilities (olmoe) */
  float resid_scale;         /* x += resid_scale * moe (1 except granitemoe) */
  float rms_eps;
} clb200_moe_layer;

typedef struct clb200_ctx clb200_ctx;

/* Opens a context on CUDA device `device` (-1: the current device). One stream per context; a context is used by one host
 * thread at a time, like the reference's single forward thread. */
clb200_ctx *clb200_open(int device, char *err, size_t errlen);
void clb200_close(clb200_ctx *c);

/* The MoE block for T tokens (1 <= T <= 512, the reference's CL_PS_B) with HOST pointers: x [T x n_embd] is read and updated
 * in place (x += resid_scale * moe); sel_out / wt_out [T x n_used] (may be NULL) receive each token's chosen experts, best
 * first, and their weights, as cl_fwd_route does (c/src/forward.h:94). Synchronous. The layer's weights are uploaded to the
 * device on first use and kept, keyed by the host pointers (they must stay valid and unchanged, as the reference's mapped
 * model does). Replaces c/src/forward.c:949-1033 (T = 1) and :1132-1210 (T > 1). */
int clb200_moe_ffn(clb200_ctx *c, const clb200_moe_layer *L, float *x, int T, int *sel_out, float *wt_out, char *err,
                   size_t errlen);

/* Device-resident use (no host copies): registers a layer and returns a handle >= 0 (or -1 with err set). With on_device = 1
 * every pointer in L is a device pointer and is used in place (the caller keeps the memory alive); with on_device = 0 the
 * tensors are copied to the device now. */
int clb200_layer_bind(clb200_ctx *c, const clb200_moe_layer *L, int on_device, char *err, size_t errlen);
/* Frees a layer's device copy (when clb200 made one) and forgets it; its handle becomes invalid. 0 on success, 1 for an
 * unknown handle. clb200_moe_ffn also drops an upload by itself when the host memory it came from no longer holds the same
 * tensors (it compares shapes and the first and last bytes of each tensor on every call). */
int clb200_layer_release(clb200_ctx *c, int layer);
/* Same block as clb200_moe_ffn on a bound layer with DEVICE pointers x [T x n_embd] (updated in place), sel [T x n_used] and
 * wt [T x n_used] (either may be NULL). Asynchronous on `stream` (a cudaStream_t; NULL: the context's stream). Argument errors
 * are reported at once; device-side errors (a timed-out wait) by clb200_status. Safe to capture in a CUDA graph once the
 * context's scratch has been sized by an earlier call with the same or larger T. */
int clb200_moe_ffn_dev(clb200_ctx *c, int layer, float *x, int T, int *sel, float *wt, void *stream, char *err,
                       size_t errlen);
/* Switches of a context (0 on success, 1 for an unknown option or value). No counterpart in the reference.
 *   CLB200_OPT_DECODE_KERNEL: which kernel runs the one-token block. 0: the expert-group kernel wherever the layer's shape
 *     allows it (each chosen expert streamed by its own group of SMs; no grid-wide wait after the routing); 1 (default): the
 *     grid-wide kernel (every SM streams a share of every chosen expert), which the expert store's calls use in any case.
 *     Both give the same results.
 *   CLB200_OPT_TEST_SPECULATION_MISS: a test hook. 1: both one-token kernels, and the whole-model step of models opened on
 *     the context, first fetch the expert ranked K + 1 in place of the one ranked K, as if two probabilities had tied at
 *     rank K, so that their correction paths run on every call (every layer); the results must not change. 0 (default):
 *     off.
 *   CLB200_OPT_TEST_STALL_WAIT: a test hook for the failure path. N > 0: the grid-wide kernel's wait for the router logits
 *     targets a count that no CTA reaches and gives up after N polls (1 << 14 is about a millisecond), so every CTA takes its
 *     error path and the launch ends with the device error word set (ERR_WAIT_ROUTER, reported by clb200_status or the host
 *     call) instead of a hang; 0 (default): off.
 *   CLB200_OPT_COOPERATIVE: 1 (default): the one-token kernels are launched cooperatively, so the driver places every CTA
 *     at once or refuses the launch (their CTAs wait on one another). 0: plain launches, one CTA per SM, which costs less per
 *     launch; for hosts that own the whole device (no other kernel can hold an SM while a launch starts). Either way a CTA
 *     that waits too long ends the launch with a device error, not a hang. */
enum { CLB200_OPT_DECODE_KERNEL = 1, CLB200_OPT_TEST_SPECULATION_MISS = 2, CLB200_OPT_TEST_STALL_WAIT = 3, CLB200_OPT_COOPERATIVE = 4 };
int clb200_set_option(clb200_ctx *c, int option, int value);
/* No counterpart in the reference: an entry point for hosts that cannot allocate device memory once they run (their
 * device memory is carved out up front by another allocator, or cudaMalloc's device-wide synchronisation would break a
 * decode latency budget). The one-token block of clb200_moe_ffn_dev on DEVICE pointers (layer tensors, x [n_embd]
 * updated in place, sel / wt [n_used] or NULL) on `stream` (NULL: the default stream), with no context: its scratch is a
 * fixed 66,560-byte array that every device holds from the time the library is loaded, and it calls no cudaMalloc,
 * cudaFree or allocating routine. Limits: K-quant expert weights, at most 128 experts, at most 16 used, and
 * n_used * n_ff_exp <= 16384; larger layers are refused with a message. The first call on a device locates the array and
 * sets the kernel's shared-memory limit on that device (make it before any stream capture). Synchronous: it returns after
 * the kernel, with the device's error word read. Every call shares the one array, so calls that overlap on the GPU (from
 * several host threads or streams) race; serialise them. The array's address is looked up once per device and kept, so do
 * not use this entry point across a cudaDeviceReset. The layer is checked as clb200_layer_bind checks it (widths 256..4096,
 * gate and up of one type, slab sizes) before anything is launched. 0 on success, 1 with err set otherwise. */
int clb200_moe_ffn_decode_noalloc(const clb200_moe_layer *L, float *x, int *sel_out, float *wt_out, void *stream, char *err,
                                  size_t errlen);
/* The dispatch step of the batched block on its own (c/src/forward.c:1162-1163 and :1188-1189), on DEVICE pointers: the
 * routing of T tokens, sel / wt [T x n_used] (expert ids, -1 never), becomes the reference's per-expert work lists.
 * todo [n_expert + 1] receives the experts that have tokens in order of first appearance in sel (the reference's todo[])
 * and, at todo[n_expert], how many there are; offsets [n_expert + 1] the start of expert e's entries in pos_token / pos_wt
 * [T x n_used] (offsets[n_expert] = the total), which hold its tokens in ascending order and their routing weights (the
 * reference's who[] / wgt[] for that expert). T up to 32768 (while n_expert x T / 32 words fit one CTA's shared memory).
 * Asynchronous on `stream` (NULL: the context's stream); an expert id out of range is reported by clb200_status. */
int clb200_moe_dispatch(clb200_ctx *c, int T, int n_expert, int n_used, const int *sel, const float *wt, int *todo,
                        int *offsets, int *pos_token, float *pos_wt, void *stream, char *err, size_t errlen);
/* ---- expert parallelism: the two halves of the batched block, around an exchange ------------------------------------------
 * No single counterpart in the reference (it runs on one machine); together with an all-to-all they are its batched block
 * (c/src/forward.c:1132-1210) with the experts spread over GPUs. Asynchronous on `stream`; K-quant gate/up experts; T up to
 * 32768. */
/* Source side of a bound layer: rmsnorm, Q8_K of xn (xq_qs [T x n_embd] int8, xq_d [T x n_embd/256] fp32, xq_bs
 * [T x n_embd/16] int16: the reference's cl_q8k rows as planes, c/src/quant.h:22), router, softmax, top-k, renormalisation
 * (sel / wt [T x n_used]) -- c/src/forward.c:1135-1155. All DEVICE pointers. */
int clb200_ep_route(clb200_ctx *c, int layer, float *x, int T, int *sel, float *wt, int8_t *xq_qs, float *xq_d, int16_t *xq_bs,
                    void *stream, char *err, size_t errlen);
/* Expert side: `layer` is a bound layer holding only this GPU's experts (n_expert = the local count); for T received rows
 * (Q8_K planes as above) with sel [T x n_used] local expert ids, -1 where the expert is another GPU's, and wt the routing
 * weights, partial [T x n_embd] = sum over the present experts, in order of first appearance, of wt * expert(row)
 * (c/src/forward.c:1160-1208 without the residual add). All DEVICE pointers. */
int clb200_ep_experts(clb200_ctx *c, int layer, int T, const int8_t *xq_qs, const float *xq_d, const int16_t *xq_bs, const int *sel,
                      const float *wt, float *partial, void *stream, char *err, size_t errlen);
/* The exchange between those two halves on the device (no reference counterpart). clb200_ep_pack: the rows each of T tokens
 * sends -- once to every one of n_ranks ranks (of n_local experts each) that holds one of its experts -- into send
 * ([T * n_ranks] rows of E + E/64 + E/8 + 8 * n_used bytes: Q8_K qs, d and bsums, the expert ids made local to the
 * destination with -1 elsewhere, the weights), ranks in order and tokens ascending within a rank; slot [T * n_ranks]: the
 * send row of (token, rank) or -1; counts [n_ranks]: the rows for each rank (device memory; the all-to-all wants them on
 * the host). clb200_ep_combine: x [T, E] += resid_scale * the sum over ranks, in rank order, of back[slot] (the partial
 * sums returned in send order). Both asynchronous on stream. */
int clb200_ep_pack(clb200_ctx *c, int T, int E, int n_used, int n_ranks, int n_local, const int *sel, const float *wt, const int8_t *xq_qs,
                   const float *xq_d, const int16_t *xq_bs, uint8_t *send, int *slot, int *counts, void *stream, char *err,
                   size_t errlen);
int clb200_ep_combine(clb200_ctx *c, int T, int E, int n_ranks, const int *slot, const float *back, float *x, float resid_scale,
                      void *stream, char *err, size_t errlen);
/* The same exchange over peer memory (NVLink / NVSwitch) instead of a library all-to-all, with no host synchronisation:
 * every rank allocates an exchange buffer of one layout (clb200_ep_xbuf_alloc: zeroed device memory and its CUDA IPC
 * handle, 64 bytes, for the other processes) and maps every other rank's (clb200_ep_xbuf_open); bufs[r] below is rank r's
 * buffer as this GPU addresses it (this rank's own at bufs[me]). clb200_ep_push stores the send rows of clb200_ep_pack
 * (counts[r] rows for rank r, device memory) into region me of each rank's receive area and then signals each with
 * (seq, rows); clb200_ep_wait (which 0) waits for every sender's signal of step seq and writes the row counts
 * (counts_out [n_ranks], device memory); region s of the receive area (clb200_ep_xbuf_layout: recv_off, n_ranks x t_max
 * rows) then holds sender s's rows in [0, counts_out[s]). clb200_ep_push_back returns the partial sums of those rows
 * (partial: [n_ranks x t_max] rows of E floats in the same regions) to each sender's back area and signals it;
 * clb200_ep_wait (which 1) waits for every rank's; clb200_ep_combine_regions is clb200_ep_combine over the back area
 * (back_off; row r * t_max + i is the i-th row sent to rank r). A rank must not push step seq + 1 before its wait for the
 * partial sums of step seq returned. Every wait is bounded: a rank that does not arrive sets the device error word
 * (clb200_status), it does not hang. All asynchronous on stream. */
void clb200_ep_xbuf_layout(int n_ranks, int t_max, int E, int n_used, size_t *bytes, size_t *recv_off, size_t *back_off);
int clb200_ep_xbuf_alloc(clb200_ctx *c, int n_ranks, int t_max, int E, int n_used, void **buf, void *ipc_handle, char *err,
                         size_t errlen);
int clb200_ep_xbuf_open(clb200_ctx *c, const void *ipc_handle, void **peer, char *err, size_t errlen);
int clb200_ep_xbuf_close(clb200_ctx *c, void *peer, char *err, size_t errlen);
int clb200_ep_xbuf_free(clb200_ctx *c, void *buf, char *err, size_t errlen);
int clb200_ep_push(clb200_ctx *c, int me, int n_ranks, int t_max, int E, int n_used, void *const *bufs, const uint8_t *send,
                   const int *counts, unsigned int seq, void *stream, char *err, size_t errlen);
int clb200_ep_wait(clb200_ctx *c, const void *own_buf, int n_ranks, int which, unsigned int seq, int *counts_out, void *stream,
                   char *err, size_t errlen);
int clb200_ep_push_back(clb200_ctx *c, int me, int n_ranks, int t_max, int E, int n_used, void *const *bufs, const float *partial,
                        const int *rcounts, unsigned int seq, void *stream, char *err, size_t errlen);
int clb200_ep_combine_regions(clb200_ctx *c, int T, int E, int n_ranks, int t_max, const int *slot, const int *counts,
                              const float *back, float *x, float resid_scale, void *stream, char *err, size_t errlen);
/* Waits for the context's work and reports a device-side error recorded since the last call (0: none). */
int clb200_status(clb200_ctx *c, char *err, size_t errlen);
/* Bytes of device memory the context holds for layers and scratch. */
uint64_t clb200_device_bytes(const clb200_ctx *c);
/* Phase trace of the one-token kernel, the device-side counterpart of the reference's CLUTOR_PROFILE phase clock
 * (c/src/forward.c:360-376): with dev_buf set (device memory, 32 uint64 per SM), every later one-token launch has thread 0 of
 * each CTA write the SM cycle counter at its phase boundaries (entries 0-29 of its row) and the global nanosecond timer at
 * entry and exit (entries 30, 31). NULL turns it off. */
void clb200_set_trace(clb200_ctx *c, void *dev_buf);
/* on = 1: batched calls (T > 1, and the batched prompt path of a model opened on this context) compute every expert product
 * on the integer path, which gives the reference's numbers bit for bit; on = 0 (the default): Q8_0 and Q4_K expert products
 * run on the tensor cores from fp16 hi/lo operands, within ~2e-5 of them and several times faster. */
void clb200_set_exact(clb200_ctx *c, int on);

/* ---- the expert cache policy (host) -------------------------------------------------------------------------------------- */
/* Which expert occupies which HBM slot: the reference's cl_cache (c/src/cache.h:11-47, c/src/cache.c), same decisions, same
 * slot numbers for the same sequence of calls. It holds no data; the device store below owns the slots. */
enum { CLB200_LRU = 0, CLB200_WTINYLFU = 1, CLB200_ADAPTIVE = 2 };                          /* cl_policy (cache.h:11) */
enum { CLB200_SEG_FREE = 0, CLB200_SEG_WINDOW, CLB200_SEG_PROBATION, CLB200_SEG_PROTECTED, CLB200_SEG_STAGE }; /* cl_list */
typedef struct {   /* cl_cache_stats (cache.h:14-17), same layout */
  uint64_t hits, misses, stage_hits, inserts, evictions, admit_rejects, stage_inserts, stage_wasted, aging_resets;
  uint32_t window_slots;
} clb200_cache_stats;
typedef struct clb200_cache clb200_cache;
/* cl_cache_new (cache.c:86-112): cache_slots experts, stage_slots prefetch slots, keys 0..universe-1 (layer * n_expert +
 * expert); window_pct 0 = the default window. NULL for zero slots or keys. */
clb200_cache *clb200_cache_new(uint32_t cache_slots, uint32_t stage_slots, uint32_t universe, int policy, uint32_t window_pct);
void clb200_cache_free(clb200_cache *c);                                   /* cl_cache_free */
uint32_t clb200_cache_total_slots(const clb200_cache *c);                  /* cl_cache_total_slots: cache + stage + 1 */
int clb200_cache_find(const clb200_cache *c, uint32_t key);                /* cl_cache_find: slot or -1 */
int clb200_cache_segment(const clb200_cache *c, int slot);                 /* cl_cache_list */
uint32_t clb200_cache_slot_key(const clb200_cache *c, int slot);           /* cl_cache_slot_key */
/* cl_cache_access (cache.c:190-216): 1 hit, 2 hit in staging (adopted), 0 miss (slot assigned and pinned: fill it),
 * -1 miss with nothing evictable (bypass). The slot is pinned in every case but -1. */
int clb200_cache_access(clb200_cache *c, uint32_t key, int *slot);
int clb200_cache_stage(clb200_cache *c, uint32_t key);                     /* cl_cache_stage (cache.c:218-232) */
void clb200_cache_pin(clb200_cache *c, int slot);                          /* cl_cache_pin */
void clb200_cache_unpin(clb200_cache *c, int slot);                        /* cl_cache_unpin */
void clb200_cache_abandon(clb200_cache *c, int slot);                      /* cl_cache_abandon */
uint32_t clb200_cache_freq(const clb200_cache *c, uint32_t key);           /* cl_cache_freq: sketch estimate 0..15 */
clb200_cache_stats clb200_cache_get_stats(const clb200_cache *c);          /* cl_cache_get_stats */
uint32_t clb200_cache_count(const clb200_cache *c);                        /* cl_cache_count: experts cached (not staged) */

/* ---- the HBM expert store ------------------------------------------------------------------------------------------------- */
/* The reference's expert store (c/src/xs.h:11-38, c/src/xs.c) with HBM slots in place of RAM slots and pinned host memory in
 * place of the model file: every layer's experts are held in pinned host memory; the cache policy above keeps a budget of
 * them in HBM slots (plus staging slots for prefetches); a miss or prefetch is one host-to-device copy on the store's copy
 * stream, overlapping the compute stream. One-token (decode) use, K-quant experts. */
typedef struct {   /* cl_xs_stats (xs.h:14-17); copy_ns = time the copy engine spent filling slots (cl_xs_stats.read_ns) */
  uint64_t accesses, hits, stage_hits, misses, bypass, prefetch_issued, prefetch_late, prefetch_wasted, admit_rejects, evictions;
  uint64_t demand_bytes, prefetch_bytes, copy_ns, wait_ns;
  uint64_t pred_total, pred_hit;   /* clb200_moe_ffn_stored: experts staged for a layer, and how many of them its router chose
                                      (the forward pass's pred_total / pred_hit, c/src/forward.h:63) */
} clb200_store_stats;
typedef struct clb200_store clb200_store;
/* cl_xs_open (xs.c:89-120): n_layer layers shaped like `shape`, HBM slots for cache_bytes (at least n_used slots), stage_slots
 * prefetch slots, policy CLB200_LRU / WTINYLFU / ADAPTIVE. Allocates n_layer * n_expert expert slots of pinned host memory.
 * NULL with err set on failure. */
clb200_store *clb200_store_open(clb200_ctx *c, const clb200_moe_layer *shape, int n_layer, uint64_t cache_bytes, int stage_slots,
                                int policy, char *err, size_t errlen);
void clb200_store_close(clb200_store *s);                                         /* cl_xs_close */
/* Copies layer `layer`'s tensors into the store (L's pointers may be host or device memory; L must have the store's shape):
 * norm and router to HBM, the experts to pinned host memory. A layer is served once loaded. */
int clb200_store_load_layer(clb200_store *s, int layer, const clb200_moe_layer *L, char *err, size_t errlen);
uint32_t clb200_store_cache_slots(const clb200_store *s);                         /* cl_xs_cache_slots */
uint64_t clb200_store_slot_bytes(const clb200_store *s);                          /* cl_xs_slot_bytes */
int clb200_store_request(clb200_store *s, int layer, int expert);                 /* cl_xs_request: handle (>= 0) or -1 */
const void *clb200_store_wait(clb200_store *s, int handle);                       /* cl_xs_wait: the expert's DEVICE address */
void clb200_store_release(clb200_store *s, int handle, void *stream);             /* cl_xs_release, once `stream`'s work so far is done */
int clb200_store_resident(clb200_store *s, int layer, int expert);                /* cl_xs_resident */
void clb200_store_prefetch(clb200_store *s, int layer, int expert);               /* cl_xs_prefetch */
clb200_store_stats clb200_store_get_stats(const clb200_store *s);                 /* cl_xs_get_stats */
void clb200_store_reset_stats(clb200_store *s);                                   /* cl_xs_reset_stats */
/* The prefetch mode of clb200_moe_ffn_stored (the reference's --prefetch, c/src/chat.c:229): 0 off; 1 (prev, the default)
 * stages the next layer's experts as the previous token chose them (c/src/forward.c:889, :894); 2 (ahead) applies the next
 * layer's norm and router to this layer's x inside the routing launch and stages its top prefetch_n experts
 * (c/src/forward.c:937-946). */
void clb200_store_set_prefetch(clb200_store *s, int mode);
/* Experts a prediction stages (--prefetch-n; 0 or >= n_used: n_used, c/src/forward.c:305). */
void clb200_store_set_prefetch_n(clb200_store *s, int n);
/* Prefetch fills in flight on the copy stream at once (default 2, at least 1): prefetch fills decided beyond that wait on the
 * host, so a demand fill queues behind at most this many (the reference's I/O queue takes demand reads first, xs.c:34-47). */
void clb200_store_set_prefetch_depth(clb200_store *s, int depth);
/* Test hooks: record every cache operation the store makes (triples: 1 access key -> code*65536+slot or -1, 2 stage key ->
 * slot, 3 unpin slot), and read the record (returns its length; copies at most cap values). */
void clb200_store_log(clb200_store *s, int on);
int64_t clb200_store_read_log(const clb200_store *s, int64_t *dst, int64_t cap);
/* A fill that fails (a copy error, or the test hook below) leaves its slot empty and makes the store failed: that wait and
 * every later one return NULL, and the stored entry points return 1 after releasing every handle of the layer, as the
 * reference's store does after a failed read (c/src/xs.c:79-80, :160-167; c/src/forward.c:1000-1001). */
int clb200_store_failed(const clb200_store *s);
/* Test hook: the n-th fill from now (n >= 1; 0 cancels) copies nothing and fails. */
void clb200_store_inject_fill_failure(clb200_store *s, int n);
/* The one-token MoE block of `layer` with its experts served by the store (c/src/forward.c:888-1033 with an expert store):
 * x [n_embd] DEVICE, updated in place; sel_out / wt_out HOST arrays [n_used] or NULL. Returns after the experts are
 * enqueued on `stream` (NULL: the context's stream); the routing is read back to the host on the way. */
int clb200_moe_ffn_stored(clb200_ctx *c, clb200_store *s, int layer, float *x, int *sel_out, float *wt_out, void *stream,
                          char *err, size_t errlen);
/* The experts of `layer` for a routing decided elsewhere (HOST sel / wt [n_used], wt renormalised), served by the store;
 * next_pred [n_used] (or NULL) are staged for layer + 1 between the requests and the waits, as the reference's stress
 * harness does with its predictor (c/src/stream.c:311-324). */
int clb200_moe_experts_stored(clb200_ctx *c, clb200_store *s, int layer, float *x, const int *sel, const float *wt,
                              const int *next_pred, void *stream, char *err, size_t errlen);

/* ---- SMART-ROUTE: cache-aware routing (c/src/route.h, c/src/route.c:13-52) ------------------------------------------------- */
typedef struct { int enabled; int J, M; double tau; } clb200_smart;   /* cl_smart (route.h:14), same layout */
typedef struct {                                                      /* cl_route_result (route.h:16-22), same layout */
  int selected[32];
  int k;
  int substituted;      /* slots filled with a different expert than the router's own choice */
  double dropped_mass;  /* sum over substitutions of (p of the expert replaced - p of the one used) */
  double max_delta;     /* largest single such difference; never exceeds tau */
} clb200_route_result;
/* cl_route (route.h:26) on the GPU, synchronous, host pointers: logits [E]; resident [E] bytes, non-zero where the expert
 * is in memory (the reference's resident callback asked for every expert), or NULL for plain routing, as is smart NULL or
 * smart->enabled 0. Returns 0; -1 when E or K is out of range (E > 1024, K > 32, K > E, or not positive), as cl_route does;
 * 1 with err set on a CUDA error. */
int clb200_route(clb200_ctx *c, const float *logits, int E, int K, const clb200_smart *smart, const uint8_t *resident,
                 clb200_route_result *out, char *err, size_t errlen);
/* The same for T tokens on device pointers, queued on `stream` (NULL: the context's): logits [T][E]; resident [E] bytes per
 * token at resident_stride (0: one set for all tokens) or NULL; out [T]. Returns 0, -1 for arguments out of range, 1 when
 * the launch fails. */
int clb200_route_dev(clb200_ctx *c, const float *logits, int T, int E, int K, const clb200_smart *smart,
                     const uint8_t *resident, int resident_stride, clb200_route_result *out, void *stream);
/* SMART-ROUTE in the store's decode step (the reference's cl_fwd_opts.smart, forward.h:100, applied at forward.c:961-969):
 * with smart->enabled, clb200_moe_ffn_stored routes on the device with the store's resident set of that layer (cl_xs_resident
 * for every expert, read when the step starts) and weights each chosen expert by its own router probability (renormalised
 * over the K where the architecture does). smart NULL or enabled 0: plain routing. Returns 0, or 1 with err set for settings
 * the reference's command line refuses (J < 0, M < 1, tau < 0; c/src/main.c:152). */
int clb200_store_set_smart(clb200_store *s, const clb200_smart *smart, char *err, size_t errlen);
typedef struct {   /* the reference's f->subs, f->expert_slots, f->dropped_mass, f->max_delta (forward.h:57-58) */
  uint64_t substituted, expert_slots;
  double dropped_mass, max_delta;
} clb200_smart_stats;
clb200_smart_stats clb200_store_smart_stats(const clb200_store *s);
/* Routing of `layer` from logits computed elsewhere (HOST, [n_expert]) against the store's resident set, as the reference's
 * stress harness routes its synthetic logits (c/src/stream.c:288-291); the choice lands in out and the store's SMART
 * counters. Synchronous. Returns 0, or 1 with err set. */
int clb200_store_route(clb200_ctx *c, clb200_store *s, int layer, const float *logits, clb200_route_result *out, char *err,
                       size_t errlen);

/* ---- the plugin seam: a cl_backend for cl_matvec_batch ------------------------------------------------------------------- */
/* Layout-compatible copies of the reference's cl_q8k, cl_xq and cl_mv (c/src/quant.h:22-34) and cl_backend (backend.h:9-13). */
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } clb200_q8k;
typedef struct { clb200_q8k *b; int n; } clb200_xq;
typedef struct {
  uint32_t type; const void *w; int rows, cols; const float *xf; const clb200_xq *xq; float *out;
  int nb; size_t xf_stride, out_stride;
} clb200_mv;
typedef struct {
  const char *name;
  int (*supports)(uint32_t type);
  void (*matvec_batch)(const clb200_mv *jobs, int n);
} clb200_backend_t;

/* The "b200" backend. supports() is 1 for Q4_K, Q6_K and Q8_0. matvec_batch() runs the jobs on the GPU (device from
 * CLUTOR_B200_DEVICE, default 0) and returns when the results are in the jobs' out arrays: K-quant jobs use the caller's
 * Q8_K activations and give the CPU's numbers bit for bit; Q8_0 jobs use the float activations in the CPU's summation order.
 * Weights are uploaded on first use, keyed by host pointer. The seam has no error channel: on a device error the backend
 * prints the error to stderr and aborts, rather than returning wrong numbers. */
const clb200_backend_t *clb200_backend(void);

/* ---- whole models: the forward pass of c/src/forward.h ------------------------------------------------------------------- */
/* A mixture-of-experts GGUF model (architectures olmoe, qwen3moe, qwen3vlmoe, granitemoe) uploaded to HBM in its own block
 * format, with a half-precision key/value cache of n_ctx positions. One token step is one persistent kernel: attention
 * (QK-norm, rotary embedding, the key/value cache), the MoE block of clb200_moe_ffn, the output matrix and the greedy
 * arg-max. Attention matrices, experts and the output matrix must be Q4_K or Q6_K; the embedding Q4_K, Q6_K, Q8_0 or F32. */
typedef struct clb200_model clb200_model;
typedef struct {
  char arch[16];
  int n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff_exp, n_expert, n_used, n_vocab, n_ctx;
  uint64_t device_bytes;   /* HBM the model holds: weights, cache, scratch */
  uint32_t smem_bytes;     /* shared memory per CTA of the step */
} clb200_model_info;
/* cl_fwd_open (forward.h:113): from a file path, or a GGUF image in host memory. n_ctx <= 0: 512 (capped at the model's). */
clb200_model *clb200_model_open(clb200_ctx *c, const char *path, int n_ctx, char *err, size_t errlen);
clb200_model *clb200_model_open_image(clb200_ctx *c, const void *image, size_t bytes, int n_ctx, char *err, size_t errlen);
void clb200_model_close(clb200_model *m);                          /* cl_fwd_close (forward.h:114) */
void clb200_model_reset(clb200_model *m);                          /* cl_fwd_reset (forward.h:115): back to position 0 */
int clb200_model_pos(const clb200_model *m);                       /* the reference's f->pos */
int clb200_model_get_info(const clb200_model *m, clb200_model_info *out);
/* cl_fwd_step (forward.h:116-117): runs `token` at the current position and advances it. logits (host, n_vocab floats),
 * next_token (the arg-max, lowest id on ties), sel_out / wt_out (host, n_layer * n_used: each layer's experts in rank order
 * and their weights, the reference's cl_fwd_route) may each be NULL. Returns 0, or 1 with err set. */
int clb200_model_step(clb200_model *m, int token, float *logits, int *next_token, int *sel_out, float *wt_out, char *err,
                      size_t errlen);
/* Greedy generation on the device, the loop of the reference's generate command (c/src/main.c:342-360) without the host:
 * feeds `token`, then each step's arg-max, n times; tokens_out (host, n) receives the n chosen tokens. */
int clb200_model_generate(clb200_model *m, int token, int n, int *tokens_out, char *err, size_t errlen);
/* The same n steps queued on `stream` (NULL: the model's own) without waiting, after one clb200_model_generate; read the
 * tokens of positions [start, start + n) afterwards with clb200_model_tokens. */
int clb200_model_generate_async(clb200_model *m, int token, int n, void *stream, char *err, size_t errlen);
int clb200_model_tokens(clb200_model *m, int start, int n, int *tokens_out, char *err, size_t errlen);
/* cl_fwd_prefill (forward.h:121, c/src/forward.c:1256-1282): feeds n tokens at the current position in batches (run_std,
 * :1078-1225): every dense matrix is multiplied with the whole batch, each token routes as it would alone and each chosen
 * expert runs once over the tokens that chose it; the attention of each token sees the positions up to its own. logits
 * (host, n_vocab floats) may be NULL, else it receives the distribution after the last token. A batch of one token is a
 * step, as in the reference. Returns 0, or 1 with err set. */
int clb200_model_prefill(clb200_model *m, const int *tokens, int n, float *logits, char *err, size_t errlen);
/* Tokens per batch of clb200_model_prefill, 1..512 (the reference's CLUTOR_PS_B; default 64, its batch for a model held in
 * memory, c/src/forward.c:1048). Returns 0, or 1 for a value out of range. */
int clb200_model_set_batch(clb200_model *m, int tokens);

#ifdef __cplusplus
}
#endif
#endif
