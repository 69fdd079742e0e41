// The HBM expert store: the reference's disk-backed expert store (c/src/xs.c, cl_xs_*) turned into a B200 memory
// hierarchy. Every layer's experts live in pinned host memory (gate, up and down slabs of one expert back to back, the
// layout of a reference slot); a budget of HBM slots holds the experts the cache policy (cache.cpp, the reference's
// cache.c) keeps, plus staging slots for prefetches and a few bypass buffers. A miss or a prefetch is one cudaMemcpyAsync
// on the store's own copy stream (a copy engine), ordered after the last kernel that read the slot's previous expert
// (an event recorded at release), so copies overlap the compute stream. cl_xs_wait's blocking wait becomes a host wait
// on the fill's event, timed, so the store reports how much of the copy time the prefetches hid.
//
// One decode step of a layer through the store (clb200_moe_ffn_stored) follows the reference's forward pass
// (c/src/forward.c:888-1033 with an expert store): stage the next layer's experts as the previous token chose them, route
// (the one-token kernel in routing mode; its choice comes back to the host), request the chosen experts resident ones first
// (c/src/forward.c:992-997), wait, run the experts from their slots (the one-token kernel in given-routing mode), release.
// Prefetch modes follow the reference's --prefetch: 1 (prev) stages the next layer's experts as the previous token chose
// them (c/src/forward.c:889, :894); 2 (ahead) applies the next layer's norm and router to this layer's x inside the same
// routing launch and stages its top prefetch_n (c/src/forward.c:937-946).
//
// Copies: demand fills go on the copy stream at once; prefetch fills wait on the host until fewer than `depth` prefetch
// fills are in flight, so a demand fill queues behind at most that many (the reference's I/O workers take every demand read
// before any prefetch read, c/src/xs.c:34-47). A demand for an expert whose prefetch is still waiting sends it at once.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <vector>

#include "ctx.cuh"
#include "route.cuh"

using namespace clb;

namespace {
enum { S_EMPTY = 0, S_LOADING = 1, S_READY = 2 };
// the SMART-ROUTE block of the store: residency, counters, logits, result
constexpr size_t SMART_RES = 0, SMART_STATS = 256, SMART_LOGITS = 512, SMART_OUT = SMART_LOGITS + 4 * 1024,
                 SMART_HOST_BYTES = SMART_OUT + 256;
uint64_t now_ns() {
  return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch()).count());
}
}  // namespace

struct clb200_store {
  clb200_ctx *ctx = nullptr;
  int n_layer = 0, NE = 0, K = 0;
  clb200_moe_layer shape{};              // widths, types and slabs every layer shares
  uint64_t expert_bytes = 0, stride = 0;
  std::vector<clb200_moe_layer> layer;   // per layer: norm and router on the device; expert pointers unused
  std::vector<uint8_t> loaded;
  uint8_t *host = nullptr;               // pinned: [layer][expert] at `stride`
  uint8_t *arena = nullptr;              // HBM: total + nbypass slots at `stride`
  uint8_t *dense = nullptr;              // HBM: every layer's norm and router
  clb200_cache *cache = nullptr;
  uint32_t total = 0, nbypass = 0, bypass_next = 0;
  std::vector<int> state;
  std::vector<cudaEvent_t> started, filled, used;
  std::vector<uint8_t> used_set, timed;
  std::vector<int> staged;               // staging slots whose fill is in flight: unpinned when it lands
  cudaStream_t copy = nullptr;
  int *sel_host = nullptr;               // pinned, device-visible: the routing kernel's choice
  float *wt_host = nullptr;
  // SMART-ROUTE: settings, counters, and a pinned device-visible block: the residency of the layer being routed [256
  // bytes], the routing kernel's counters (RouteStats), logits handed in by the host [1024 floats], a routing result
  uint8_t *smart_host = nullptr;
  clb200_smart smart{};
  clb200_smart_stats smart_st{};
  std::vector<int> prev_sel;             // [n_layer * K] the previous token's choice, -1 before the first
  std::vector<int> pred_sel;             // [n_layer * K] what was staged for this token's layer, -1 for none
  int prefetch = 1;                      // 0 off, 1 prev, 2 ahead
  int prefetch_n = 0;                    // experts a prediction stages (0: n_used)
  int depth = 2;                         // prefetch fills on the copy stream at once
  struct Pending { int buf, layer, expert; };
  std::vector<Pending> pending;          // prefetch fills decided, not yet on the copy stream (oldest first)
  int *ahead_host = nullptr;             // pinned, device-visible: router-ahead's choice
  clb200_store_stats st{};
  uint64_t dev_bytes = 0;                // device memory counted in the context's total
  bool logging = false;
  std::vector<int64_t> oplog;
  // a fill that failed makes every later wait fail (the reference's sticky failed flag, c/src/xs.c:79, :160); fail_in > 0:
  // test hook, the fail_in-th fill from now does not copy and fails
  bool failed = false;
  int fail_in = 0;
  std::vector<uint8_t> fill_failed;
};

namespace {

void log_op(clb200_store *s, int op, int64_t a, int64_t r) {
  if (s->logging) {
    s->oplog.push_back(op);
    s->oplog.push_back(a);
    s->oplog.push_back(r);
  }
}

// The reference's SMART counters (c/src/forward.c:968-969): substitutions and probability moved, summed; the largest delta.
void count_smart(clb200_store *s, const RouteStats &r) {
  s->smart_st.substituted += static_cast<uint64_t>(r.substituted);
  s->smart_st.dropped_mass += r.dropped_mass;
  if (r.max_delta > s->smart_st.max_delta) s->smart_st.max_delta = r.max_delta;
}

void count_copy(clb200_store *s, int buf) {   // the fill of `buf` has completed: add its duration to copy_ns once
  if (s->timed[buf]) return;
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, s->started[buf], s->filled[buf]) == cudaSuccess) s->st.copy_ns += static_cast<uint64_t>(ms * 1e6);
  s->timed[buf] = 1;
}

void fill(clb200_store *s, int buf, int layer, int expert, bool prefetch);

// Prefetch fills go on the copy stream while fewer than `depth` are in flight there.
void pump(clb200_store *s) {
  size_t i = 0;
  while (i < s->pending.size() && static_cast<int>(s->staged.size()) < s->depth) {
    const clb200_store::Pending p = s->pending[i++];
    fill(s, p.buf, p.layer, p.expert, true);
    s->staged.push_back(p.buf);
  }
  s->pending.erase(s->pending.begin(), s->pending.begin() + static_cast<long>(i));
}

// A prefetch of `buf` still waiting on the host goes on the copy stream now (a demand needs it); false if none waits.
bool promote(clb200_store *s, int buf) {
  for (size_t i = 0; i < s->pending.size(); ++i)
    if (s->pending[i].buf == buf) {
      const clb200_store::Pending p = s->pending[i];
      s->pending.erase(s->pending.begin() + static_cast<long>(i));
      fill(s, p.buf, p.layer, p.expert, true);
      s->staged.push_back(p.buf);
      return true;
    }
  return false;
}

// Staging fills that have landed: ready, and unpinned (the reference's I/O worker does this when a prefetch read ends);
// then waiting prefetch fills take the places freed.
void poll(clb200_store *s) {
  size_t keep = 0;
  for (size_t i = 0; i < s->staged.size(); ++i) {
    const int b = s->staged[i];
    if (cudaEventQuery(s->filled[b]) == cudaSuccess) {
      if (s->fill_failed[b]) {   // a failed read leaves the slot empty (c/src/xs.c:79-80)
        s->fill_failed[b] = 0;
        s->failed = true;
        s->state[b] = S_EMPTY;
      } else {
        s->state[b] = S_READY;
        count_copy(s, b);
      }
      clb200_cache_unpin(s->cache, b);
      log_op(s, 3, b, 0);
    } else {
      s->staged[keep++] = b;
    }
  }
  s->staged.resize(keep);
  cudaGetLastError();   // a "not ready" answer is not an error
  pump(s);
}

// cl_xs_resident (c/src/xs.c:179-186) for every expert of `layer`, into the pinned residency bytes the kernels read.
void fill_resident(clb200_store *s, int layer) {
  poll(s);
  for (int e = 0; e < s->NE; ++e) {
    const int slot = clb200_cache_find(s->cache, static_cast<uint32_t>(layer * s->NE + e));
    s->smart_host[SMART_RES + e] = static_cast<uint8_t>(slot >= 0 && s->state[slot] == S_READY);
  }
}

void fill(clb200_store *s, int buf, int layer, int expert, bool prefetch) {
  if (s->used_set[buf]) cudaStreamWaitEvent(s->copy, s->used[buf], 0);   // the previous expert's readers are done
  cudaEventRecord(s->started[buf], s->copy);
  if (s->fail_in > 0 && --s->fail_in == 0) {   // test hook: this fill reads nothing and fails
    s->fill_failed[buf] = 1;
  } else {
    cudaMemcpyAsync(s->arena + static_cast<size_t>(buf) * s->stride,
                    s->host + (static_cast<size_t>(layer) * s->NE + expert) * s->stride, s->expert_bytes, cudaMemcpyHostToDevice, s->copy);
  }
  cudaEventRecord(s->filled[buf], s->copy);
  s->state[buf] = S_LOADING;
  s->timed[buf] = 0;
  (prefetch ? s->st.prefetch_bytes : s->st.demand_bytes) += s->expert_bytes;
}

bool valid_expert(const clb200_store *s, int layer, int expert) {
  return s && layer >= 0 && layer < s->n_layer && expert >= 0 && expert < s->NE && s->loaded[layer];
}

}  // namespace

extern "C" {

clb200_store *clb200_store_open(clb200_ctx *c, const clb200_moe_layer *shape, int n_layer, uint64_t cache_bytes, int stage_slots,
                                int policy, char *err, size_t errlen) {
  if (!c || !shape || n_layer < 1) { errf(err, errlen, "no context, shape or layers"); return nullptr; }
  if (validate(shape, err, errlen)) return nullptr;
  DecodeArgs probe{};
  if (plan_decode_shape(c->sms, c->max_smem, *shape, probe)) { errf(err, errlen, "the store serves the one-token kernel: K-quant experts only"); return nullptr; }
  cudaSetDevice(c->device);
  auto *s = new clb200_store();
  s->ctx = c;
  s->n_layer = n_layer;
  s->NE = shape->n_expert;
  s->K = shape->n_used;
  s->shape = *shape;
  s->expert_bytes = shape->gate_slab + shape->up_slab + shape->down_slab;
  s->stride = al(s->expert_bytes, 256);
  s->layer.assign(n_layer, *shape);
  s->loaded.assign(n_layer, 0);
  s->prev_sel.assign(static_cast<size_t>(n_layer) * s->K, -1);
  s->pred_sel.assign(static_cast<size_t>(n_layer) * s->K, -1);
  uint32_t slots = static_cast<uint32_t>(cache_bytes / s->stride);
  if (slots < static_cast<uint32_t>(s->K)) slots = static_cast<uint32_t>(s->K);   // a layer's experts must fit at once (xs.c:103)
  s->cache = clb200_cache_new(slots, stage_slots < 0 ? 0u : static_cast<uint32_t>(stage_slots),
                              static_cast<uint32_t>(n_layer) * static_cast<uint32_t>(s->NE), policy, 0);
  if (!s->cache) { errf(err, errlen, "bad cache settings"); delete s; return nullptr; }
  s->total = clb200_cache_total_slots(s->cache);
  s->nbypass = static_cast<uint32_t>(s->K) + 2;
  const uint32_t nbuf = s->total + s->nbypass;
  const size_t host_bytes = static_cast<size_t>(n_layer) * s->NE * s->stride;
  const size_t dense_per = al(static_cast<size_t>(shape->n_embd) * 4) + al(static_cast<size_t>(s->NE) * shape->n_embd * 4);
  bool ok = cudaHostAlloc(reinterpret_cast<void **>(&s->host), host_bytes, cudaHostAllocDefault) == cudaSuccess &&
            cudaMalloc(&s->arena, static_cast<size_t>(nbuf) * s->stride) == cudaSuccess &&
            cudaMalloc(&s->dense, dense_per * n_layer) == cudaSuccess &&
            cudaHostAlloc(reinterpret_cast<void **>(&s->sel_host), 64 * sizeof(int), cudaHostAllocMapped) == cudaSuccess &&
            cudaHostAlloc(reinterpret_cast<void **>(&s->wt_host), 64 * sizeof(float), cudaHostAllocMapped) == cudaSuccess &&
            cudaHostAlloc(reinterpret_cast<void **>(&s->smart_host), SMART_HOST_BYTES, cudaHostAllocMapped) == cudaSuccess &&
            cudaHostAlloc(reinterpret_cast<void **>(&s->ahead_host), 64 * sizeof(int), cudaHostAllocMapped) == cudaSuccess &&
            cudaStreamCreateWithFlags(&s->copy, cudaStreamNonBlocking) == cudaSuccess;
  s->state.assign(nbuf, S_EMPTY);
  s->fill_failed.assign(nbuf, 0);
  s->used_set.assign(nbuf, 0);
  s->timed.assign(nbuf, 1);
  s->started.assign(nbuf, nullptr);
  s->filled.assign(nbuf, nullptr);
  s->used.assign(nbuf, nullptr);
  for (uint32_t i = 0; ok && i < nbuf; ++i)
    ok = cudaEventCreate(&s->started[i]) == cudaSuccess && cudaEventCreate(&s->filled[i]) == cudaSuccess &&
         cudaEventCreateWithFlags(&s->used[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    errf(err, errlen, "cannot allocate the store: %zu bytes pinned host memory and %zu bytes on device %d", host_bytes,
         static_cast<size_t>(nbuf) * s->stride + dense_per * n_layer, c->device);
    clb200_store_close(s);
    return nullptr;
  }
  for (int l = 0; l < n_layer; ++l) {
    s->layer[l].ffn_norm_f = reinterpret_cast<const float *>(s->dense + dense_per * l);
    s->layer[l].router_f = reinterpret_cast<const float *>(s->dense + dense_per * l + al(static_cast<size_t>(shape->n_embd) * 4));
    s->layer[l].gate.p = s->layer[l].up.p = s->layer[l].down.p = nullptr;
  }
  s->dev_bytes = static_cast<uint64_t>(nbuf) * s->stride + dense_per * n_layer;
  c->bytes += s->dev_bytes;
  return s;
}

void clb200_store_close(clb200_store *s) {
  if (!s) return;
  cudaSetDevice(s->ctx->device);
  if (s->copy) cudaStreamSynchronize(s->copy);
  cudaStreamSynchronize(s->ctx->stream);
  for (auto e : s->started) if (e) cudaEventDestroy(e);
  for (auto e : s->filled) if (e) cudaEventDestroy(e);
  for (auto e : s->used) if (e) cudaEventDestroy(e);
  if (s->copy) cudaStreamDestroy(s->copy);
  if (s->arena) cudaFree(s->arena);
  s->ctx->bytes -= s->dev_bytes;
  if (s->dense) cudaFree(s->dense);
  if (s->host) cudaFreeHost(s->host);
  if (s->sel_host) cudaFreeHost(s->sel_host);
  if (s->wt_host) cudaFreeHost(s->wt_host);
  if (s->smart_host) cudaFreeHost(s->smart_host);
  if (s->ahead_host) cudaFreeHost(s->ahead_host);
  if (s->cache) clb200_cache_free(s->cache);
  delete s;
}

int clb200_store_load_layer(clb200_store *s, int layer, const clb200_moe_layer *L, char *err, size_t errlen) {
  if (!s || layer < 0 || layer >= s->n_layer) { errf(err, errlen, "no layer %d in the store", layer); return 1; }
  if (validate(L, err, errlen)) return 1;
  const clb200_moe_layer &h = s->shape;
  if (L->n_embd != h.n_embd || L->n_ff_exp != h.n_ff_exp || L->n_expert != h.n_expert || L->n_used != h.n_used ||
      L->gate.type != h.gate.type || L->down.type != h.down.type) {
    errf(err, errlen, "layer %d does not have the store's shape", layer);
    return 1;
  }
  cudaSetDevice(s->ctx->device);
  clb200_moe_layer &d = s->layer[layer];
  const size_t E = h.n_embd, NE = h.n_expert;
  d.norm_topk = L->norm_topk;
  d.resid_scale = L->resid_scale;
  d.rms_eps = L->rms_eps;
  CUDA_OR(cudaMemcpy(const_cast<float *>(d.ffn_norm_f), L->ffn_norm_f, E * 4, cudaMemcpyDefault), "copying the norm weights");
  CUDA_OR(cudaMemcpy(const_cast<float *>(d.router_f), L->router_f, NE * E * 4, cudaMemcpyDefault), "copying the router");
  // expert e of the layer at host + (layer * NE + e) * stride: gate, up, down slabs back to back (the reference's slot layout)
  uint8_t *dst = s->host + static_cast<size_t>(layer) * NE * s->stride;
  CUDA_OR(cudaMemcpy2D(dst, s->stride, L->gate.p, h.gate_slab, h.gate_slab, NE, cudaMemcpyDefault), "copying gate experts");
  CUDA_OR(cudaMemcpy2D(dst + h.gate_slab, s->stride, L->up.p, h.up_slab, h.up_slab, NE, cudaMemcpyDefault), "copying up experts");
  CUDA_OR(cudaMemcpy2D(dst + h.gate_slab + h.up_slab, s->stride, L->down.p, h.down_slab, h.down_slab, NE, cudaMemcpyDefault),
          "copying down experts");
  s->loaded[layer] = 1;
  return 0;
}

uint32_t clb200_store_cache_slots(const clb200_store *s) { return s ? s->total : 0; }
uint64_t clb200_store_slot_bytes(const clb200_store *s) { return s ? s->stride : 0; }
void clb200_store_set_prefetch(clb200_store *s, int mode) { if (s) s->prefetch = mode < 0 ? 0 : mode > 2 ? 2 : mode; }

void clb200_store_set_prefetch_n(clb200_store *s, int n) { if (s) s->prefetch_n = n < 0 ? 0 : n; }

void clb200_store_set_prefetch_depth(clb200_store *s, int depth) { if (s) s->depth = depth < 1 ? 1 : depth; }

int clb200_store_request(clb200_store *s, int layer, int expert) {
  if (!valid_expert(s, layer, expert)) return -1;
  poll(s);
  const uint32_t key = static_cast<uint32_t>(layer * s->NE + expert);
  int slot = -1;
  const int r = clb200_cache_access(s->cache, key, &slot);
  log_op(s, 1, key, r >= 0 ? r * 65536 + slot : -1);
  ++s->st.accesses;
  if (r == 1) {
    ++s->st.hits;
  } else if (r == 2) {
    ++s->st.stage_hits;
    ++s->st.hits;
    if (s->state[slot] != S_READY) ++s->st.prefetch_late;
    promote(s, slot);
  } else {
    ++s->st.misses;
    if (r == -1) {   // nothing evictable: a bypass buffer outside the cache (xs.c:160-163)
      slot = static_cast<int>(s->total + (s->bypass_next++ % s->nbypass));
      ++s->st.bypass;
    }
    fill(s, slot, layer, expert, false);
  }
  return slot;
}

const void *clb200_store_wait(clb200_store *s, int h) {
  if (!s || h < 0 || h >= static_cast<int>(s->total + s->nbypass)) return nullptr;
  if (s->state[h] != S_READY && !s->failed) {
    poll(s);   // prefetch fills freed by landed ones join the copy stream behind this one
    const uint64_t t0 = now_ns();
    const cudaError_t e = cudaEventSynchronize(s->filled[h]);
    s->st.wait_ns += now_ns() - t0;
    if (e != cudaSuccess || s->fill_failed[h]) {   // a failed read: the slot stays empty, and so does every later wait
      s->fill_failed[h] = 0;
      s->failed = true;
      s->state[h] = S_EMPTY;
      return nullptr;
    }
    s->state[h] = S_READY;
  }
  if (s->state[h] != S_READY) return nullptr;   // the store has failed (c/src/xs.c:160-167)
  count_copy(s, h);
  return s->arena + static_cast<size_t>(h) * s->stride;
}

void clb200_store_inject_fill_failure(clb200_store *s, int n) {
  if (s) s->fail_in = n > 0 ? n : 0;
}

int clb200_store_failed(const clb200_store *s) { return s && s->failed ? 1 : 0; }

void clb200_store_release(clb200_store *s, int h, void *stream) {
  if (!s || h < 0 || h >= static_cast<int>(s->total + s->nbypass)) return;
  cudaEventRecord(s->used[h], stream ? static_cast<cudaStream_t>(stream) : s->ctx->stream);   // the next fill waits for it
  s->used_set[h] = 1;
  if (static_cast<uint32_t>(h) < s->total) {
    clb200_cache_unpin(s->cache, h);
    log_op(s, 3, h, 0);
  } else {
    s->state[h] = S_EMPTY;
  }
}

int clb200_store_resident(clb200_store *s, int layer, int expert) {
  if (!valid_expert(s, layer, expert)) return 0;
  poll(s);
  const int slot = clb200_cache_find(s->cache, static_cast<uint32_t>(layer * s->NE + expert));
  return slot >= 0 && s->state[slot] == S_READY;
}

void clb200_store_prefetch(clb200_store *s, int layer, int expert) {
  if (!valid_expert(s, layer, expert)) return;
  poll(s);
  const uint32_t key = static_cast<uint32_t>(layer * s->NE + expert);
  const int slot = clb200_cache_stage(s->cache, key);
  log_op(s, 2, key, slot);
  if (slot < 0) return;
  s->state[slot] = S_LOADING;
  s->pending.push_back({slot, layer, expert});
  ++s->st.prefetch_issued;
  pump(s);
}

clb200_store_stats clb200_store_get_stats(const clb200_store *s) {
  clb200_store_stats r{};
  if (!s) return r;
  r = s->st;
  const clb200_cache_stats cs = clb200_cache_get_stats(s->cache);
  r.evictions = cs.evictions;
  r.admit_rejects = cs.admit_rejects;
  r.prefetch_wasted = cs.stage_wasted;
  return r;
}

void clb200_store_reset_stats(clb200_store *s) {
  if (!s) return;
  s->st = clb200_store_stats{};
  s->smart_st = clb200_smart_stats{};
}

void clb200_store_log(clb200_store *s, int on) {
  if (!s) return;
  s->logging = on != 0;
  s->oplog.clear();
}

int64_t clb200_store_read_log(const clb200_store *s, int64_t *dst, int64_t cap) {
  if (!s) return 0;
  const int64_t n = static_cast<int64_t>(s->oplog.size());
  if (dst) std::memcpy(dst, s->oplog.data(), static_cast<size_t>(n < cap ? n : cap) * sizeof(int64_t));
  return n;
}

// Experts of `layer` for one token with the routing sel / wt [n_used] given (host arrays): requests (resident ones first),
// stages next_pred [n_used] of layer + 1 when given, waits, runs the experts from their slots and releases them.
static int experts_stored(clb200_ctx *c, clb200_store *s, int layer, float *x, const int *sel, const float *wt, const int *next_pred,
                          cudaStream_t st, char *err, size_t errlen) {
  const int K = s->K;
  int h[DECODE_MAX_K];
  const uint8_t *ptr[DECODE_MAX_K];
  for (int k = 0; k < K; ++k)
    if (sel[k] < 0 || sel[k] >= s->NE) { errf(err, errlen, "expert %d out of range", sel[k]); return 1; }
  // ask for what is already in HBM first, so a miss cannot evict an expert this layer is about to use
  int here[DECODE_MAX_K];
  for (int k = 0; k < K; ++k) here[k] = clb200_store_resident(s, layer, sel[k]);
  for (int pass = 0; pass < 2; ++pass)
    for (int k = 0; k < K; ++k)
      if ((pass == 0) == (here[k] != 0)) h[k] = clb200_store_request(s, layer, sel[k]);
  if (next_pred && layer + 1 < s->n_layer && s->loaded[layer + 1])
    for (int k = 0; k < K; ++k) clb200_store_prefetch(s, layer + 1, next_pred[k]);
  for (int k = 0; k < K; ++k) {
    ptr[k] = static_cast<const uint8_t *>(clb200_store_wait(s, h[k]));
    if (!ptr[k]) {   // every handle of the layer goes back before the error (c/src/forward.c:1000-1001)
      errf(err, errlen, "reading expert %d of layer %d into HBM failed", sel[k], layer);
      for (int j = 0; j < K; ++j) clb200_store_release(s, h[j], st);
      return 1;
    }
  }
  const int rc = launch_one(c, s->layer[layer], x, 2, sel, wt, ptr, nullptr, nullptr, st, err, errlen);
  for (int k = 0; k < K; ++k) clb200_store_release(s, h[k], st);
  return rc;
}

int clb200_moe_experts_stored(clb200_ctx *c, clb200_store *s, int layer, float *x, const int *sel, const float *wt,
                              const int *next_pred, void *stream, char *err, size_t errlen) {
  if (!c || !s || s->ctx != c) { errf(err, errlen, "no context or store, or a store of another context"); return 1; }
  if (layer < 0 || layer >= s->n_layer || !s->loaded[layer]) { errf(err, errlen, "layer %d is not loaded", layer); return 1; }
  if (!x || !sel || !wt) { errf(err, errlen, "no activations or routing"); return 1; }
  cudaSetDevice(c->device);
  return experts_stored(c, s, layer, x, sel, wt, next_pred, stream ? static_cast<cudaStream_t>(stream) : c->stream, err, errlen);
}

int clb200_moe_ffn_stored(clb200_ctx *c, clb200_store *s, int layer, float *x, int *sel_out, float *wt_out, void *stream,
                          char *err, size_t errlen) {
  if (!c || !s || s->ctx != c) { errf(err, errlen, "no context or store, or a store of another context"); return 1; }
  if (layer < 0 || layer >= s->n_layer || !s->loaded[layer]) { errf(err, errlen, "layer %d is not loaded", layer); return 1; }
  if (!x) { errf(err, errlen, "no activations"); return 1; }
  cudaSetDevice(c->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  const int K = s->K, pn = s->prefetch_n > 0 && s->prefetch_n < K ? s->prefetch_n : K;
  int *pred_next = layer + 1 < s->n_layer ? s->pred_sel.data() + static_cast<size_t>(layer + 1) * K : nullptr;
  if (layer == 0) {   // a new token (c/src/forward.c:888-889): nothing predicted yet; layer 0 as the previous token chose it
    std::fill(s->pred_sel.begin(), s->pred_sel.end(), -1);
    if (s->prefetch)
      for (int k = 0; k < pn; ++k) {
        clb200_store_prefetch(s, 0, s->prev_sel[k]);
        s->pred_sel[k] = s->prev_sel[k];
      }
  }
  if (s->prefetch == 1 && pred_next)   // the next layer as the previous token chose it (c/src/forward.c:894)
    for (int k = 0; k < pn; ++k) {
      const int e = s->prev_sel[static_cast<size_t>(layer + 1) * K + k];
      clb200_store_prefetch(s, layer + 1, e);
      pred_next[k] = e;
    }
  SmartRoute sr{};
  const bool smart = s->smart.enabled != 0;
  if (smart) {   // the layer's resident set as the routing starts (c/src/forward.c:963-966 asks cl_xs_resident)
    fill_resident(s, layer);
    sr.resident = s->smart_host + SMART_RES;
    sr.J = s->smart.J;
    sr.M = s->smart.M;
    sr.tau = s->smart.tau;
    sr.stats = s->smart_host + SMART_STATS;
  }
  AheadRoute ar{};
  const bool ahead = s->prefetch == 2 && pred_next && s->loaded[layer + 1];
  if (ahead) {   // the next layer's router on this x, in the same routing launch
    ar.norm = s->layer[layer + 1].ffn_norm_f;
    ar.router = s->layer[layer + 1].router_f;
    ar.n = pn;
    ar.out = s->ahead_host;
  }
  if (launch_one(c, s->layer[layer], x, 1, nullptr, nullptr, nullptr, s->sel_host, s->wt_host, st, err, errlen, smart ? &sr : nullptr,
                 nullptr, nullptr, ahead ? &ar : nullptr))
    return 1;
  CUDA_OR(cudaStreamSynchronize(st), "routing");
  if (ahead)   // staged before this layer's requests, in the reference's order; their copies follow the demand fills
    for (int k = 0; k < pn; ++k) {
      clb200_store_prefetch(s, layer + 1, s->ahead_host[k]);
      pred_next[k] = s->ahead_host[k];
    }
  if (smart) count_smart(s, *reinterpret_cast<const RouteStats *>(s->smart_host + SMART_STATS));
  s->smart_st.expert_slots += static_cast<uint64_t>(K);
  int sel[DECODE_MAX_K];
  float wt[DECODE_MAX_K];
  for (int k = 0; k < K; ++k) {
    sel[k] = s->sel_host[k];
    wt[k] = s->wt_host[k];
    s->prev_sel[static_cast<size_t>(layer) * K + k] = sel[k];
  }
  for (int k = 0; k < pn; ++k) {   // how many staged experts the router then chose (c/src/forward.c:978-983)
    const int pe = s->pred_sel[static_cast<size_t>(layer) * K + k];
    if (pe < 0) continue;
    ++s->st.pred_total;
    for (int j = 0; j < K; ++j)
      if (sel[j] == pe) { ++s->st.pred_hit; break; }
  }
  if (experts_stored(c, s, layer, x, sel, wt, nullptr, st, err, errlen)) return 1;
  if (sel_out) std::memcpy(sel_out, sel, K * sizeof(int));
  if (wt_out) std::memcpy(wt_out, wt, K * sizeof(float));
  return 0;
}

int clb200_store_set_smart(clb200_store *s, const clb200_smart *smart, char *err, size_t errlen) {
  if (!s) { errf(err, errlen, "no store"); return 1; }
  if (!smart || !smart->enabled) {
    s->smart = clb200_smart{};
    return 0;
  }
  if (smart->J < 0 || smart->M < 1 || !(smart->tau >= 0.0)) { errf(err, errlen, "SMART-ROUTE wants J >= 0, M >= 1 and tau >= 0"); return 1; }
  if (s->NE > ROUTE_SMEM_MAX_NE || s->K > ROUTE_MAX_K) { errf(err, errlen, "SMART-ROUTE takes at most %d experts and %d used", ROUTE_SMEM_MAX_NE, ROUTE_MAX_K); return 1; }
  s->smart = *smart;
  s->smart.enabled = 1;
  return 0;
}

clb200_smart_stats clb200_store_smart_stats(const clb200_store *s) { return s ? s->smart_st : clb200_smart_stats{}; }

int clb200_store_route(clb200_ctx *c, clb200_store *s, int layer, const float *logits, clb200_route_result *out, char *err,
                       size_t errlen) {
  if (!c || !s || s->ctx != c) { errf(err, errlen, "no context or store, or a store of another context"); return 1; }
  if (layer < 0 || layer >= s->n_layer) { errf(err, errlen, "layer %d is outside the store", layer); return 1; }
  if (!logits || !out) { errf(err, errlen, "no logits or result"); return 1; }
  if (s->NE > ROUTE_MAX_E) { errf(err, errlen, "too many experts to route"); return 1; }
  cudaSetDevice(c->device);
  const bool smart = s->smart.enabled != 0;
  if (smart) fill_resident(s, layer);
  std::memcpy(s->smart_host + SMART_LOGITS, logits, static_cast<size_t>(s->NE) * 4);
  auto *res = reinterpret_cast<clb200_route_result *>(s->smart_host + SMART_OUT);
  if (launch_route_kernel(reinterpret_cast<const float *>(s->smart_host + SMART_LOGITS), 1, s->NE, s->K, smart ? &s->smart : nullptr,
                          smart ? s->smart_host + SMART_RES : nullptr, 0, res, c->stream)) {
    errf(err, errlen, "launching the routing kernel: %s", cudaGetErrorString(cudaGetLastError()));
    return 1;
  }
  CUDA_OR(cudaStreamSynchronize(c->stream), "routing");
  *out = *res;
  RouteStats r{};
  r.substituted = res->substituted;
  r.dropped_mass = res->dropped_mass;
  r.max_delta = res->max_delta;
  if (smart) count_smart(s, r);
  s->smart_st.expert_slots += static_cast<uint64_t>(s->K);
  return 0;
}

}  // extern "C"
