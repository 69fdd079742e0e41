// The C ABI of include/clb200.h: contexts, layer registration and upload, scratch, the per-layer MoE entry points and the
// "b200" cl_backend.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "ctx.cuh"

using namespace clb;


namespace clb {

struct Scratch {
  size_t off_logits, off_hg, off_x, off_sel, off_wt, total;
  // batched
  size_t off_xn, off_xq_qs, off_xq_d, off_xq_bs, off_bsel, off_bwt, off_counts, off_offsets, off_first, off_todo, off_pos_token,
      off_pos_wt, off_slot_pos, off_bhg, off_hq_qs, off_hq_d, off_hq_bs, off_hd, off_xh, off_xl, off_hgh, off_hgl, off_xdh, off_xdl, off_rs;
};

// `batched`: the batched kernels will run (T > 1, or one token of a shape the one-token kernel does not take).
static Scratch plan_scratch(int T, int E, int FF, int NE, int K, bool batched) {
  Scratch s{};
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = al(o + bytes); return at; };
  const size_t TK = static_cast<size_t>(T) * K;
  s.off_x = take(static_cast<size_t>(T) * E * 4);
  s.off_sel = take(TK * 4);
  s.off_wt = take(TK * 4);
  s.off_logits = take(static_cast<size_t>(T < 2 ? 2 : T) * NE * 4);   // one token: router-ahead's logits follow the layer's
  s.off_hg = take(static_cast<size_t>(K) * FF * 4);
  if (batched) {
    s.off_xn = take(static_cast<size_t>(T) * E * 4);
    s.off_xq_qs = take(static_cast<size_t>(T) * E);
    s.off_xq_d = take(static_cast<size_t>(T) * (E / 256) * 4);
    s.off_xq_bs = take(static_cast<size_t>(T) * (E / 16) * 2);
    s.off_bsel = take(TK * 4);
    s.off_bwt = take(TK * 4);
    s.off_counts = take(static_cast<size_t>(NE) * 4);
    s.off_offsets = take(static_cast<size_t>(NE + 1) * 4);
    s.off_first = take(static_cast<size_t>(NE) * 4);
    s.off_todo = take(static_cast<size_t>(NE + 1) * 4);
    s.off_pos_token = take(TK * 4);
    s.off_pos_wt = take(TK * 4);
    s.off_slot_pos = take(TK * 4);
    s.off_bhg = take(TK * FF * 4);
    s.off_hq_qs = take(TK * FF);
    s.off_hq_d = take(TK * (FF / 256) * 4);
    s.off_hq_bs = take(TK * (FF / 16) * 2);
    s.off_hd = take(TK * E * 4);
    s.off_xh = take(static_cast<size_t>(T) * E * 2);
    s.off_xl = take(static_cast<size_t>(T) * E * 2);
    s.off_hgh = take(TK * FF * 2);
    s.off_hgl = take(TK * FF * 2);
    s.off_xdh = take(TK * E * 2);
    s.off_xdl = take(TK * E * 2);
    s.off_rs = take(TK * 4);
  }
  s.total = o;
  return s;
}

static int ensure_scratch(clb200_ctx *c, size_t need, char *err, size_t errlen) {
  if (need <= c->scratch_cap) return 0;
  CUDA_OR(cudaStreamSynchronize(c->stream), "waiting for the device before growing scratch");
  if (c->scratch) { cudaFree(c->scratch); c->bytes -= c->scratch_cap; }
  c->scratch = nullptr;
  c->scratch_cap = 0;
  const size_t cap = al(need, 1 << 20);
  CUDA_OR(cudaMalloc(&c->scratch, cap), "allocating scratch");
  c->scratch_cap = cap;
  ++c->graph_gen;
  c->bytes += cap;
  return 0;
}

static int ensure_hstage(clb200_ctx *c, size_t need, char *err, size_t errlen) {
  if (need <= c->hstage_cap) return 0;
  if (c->hstage) {
    CUDA_OR(cudaStreamSynchronize(c->stream), "waiting for the device before growing host staging");
    cudaFreeHost(c->hstage);
  }
  c->hstage = nullptr;
  c->hstage_dev = nullptr;
  c->hstage_cap = 0;
  const size_t cap = al(need, 1 << 16);
  CUDA_OR(cudaHostAlloc(reinterpret_cast<void **>(&c->hstage), cap, cudaHostAllocMapped | cudaHostAllocPortable), "pinning host staging");
  c->hstage_cap = cap;
  CUDA_OR(cudaHostGetDevicePointer(reinterpret_cast<void **>(&c->hstage_dev), c->hstage, 0), "mapping host staging");
  ++c->graph_gen;
  return 0;
}

// Shared-memory plan of the one-token kernel for a layer on a device with `sms` SMs and `max_smem` bytes of opt-in shared
// memory per block; 0 when it fits.
int plan_decode_shape(int sms, int max_smem, const clb200_moe_layer &L, DecodeArgs &a) {
  const int G = sms, E = L.n_embd, FF = L.n_ff_exp, NE = L.n_expert, K = L.n_used;
  auto kq = [](uint32_t t) { return t == T_Q4_K || t == T_Q6_K; };
  // four threads rank each expert, one warp issues each expert's copies
  if (!kq(L.gate.type) || !kq(L.up.type) || !kq(L.down.type) || NE > DECODE_THREADS / 4 || K > DECODE_MAX_K) return 1;
  const int nb = E / 256, nbd = FF / 256;
  if (nbd * K > DECODE_THREADS || nb > DECODE_THREADS / 8 || K > DECODE_THREADS / 32) return 1;   // one warp issues each expert's copies
  a.rgu_max = (FF + G - 1) / G;
  a.rd_max = (E + G - 1) / G;
  a.grb = static_cast<uint32_t>(row_bytes(L.gate.type, E));
  a.drb = static_cast<uint32_t>(row_bytes(L.down.type, FF));
  a.gseg = static_cast<uint32_t>(al(static_cast<size_t>(a.rgu_max) * a.grb + 32, 16));
  a.dseg = static_cast<uint32_t>(al(static_cast<size_t>(a.rd_max) * a.drb + 32, 16));
  a.slot_bytes = 2 * a.gseg + a.dseg;
  a.slot_bytes += (16 - a.slot_bytes % 128 + 128) % 128;   // slots 16 bytes off a 128-byte period: experts in different banks
  const int nre = (NE + G - 1) / G;
  constexpr int NW = DECODE_THREADS / 32;
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = al(o + bytes, 16); return static_cast<uint32_t>(at); };
  a.off_bars = take(8 * (2 * K + 1));
  a.off_xn = take(static_cast<size_t>(E) * 4);
  a.off_norm = take(static_cast<size_t>(E) * 4);
  a.off_xq = take(static_cast<size_t>(E) + 2 * (E / 16) + 4 * (E / 256));
  a.off_router = take(static_cast<size_t>(nre) * E * 4);
  // products, one padded row per strided sum; later the weighted expert outputs of this CTA's rows, [rd_max][K]
  a.off_rprod = take(std::max(static_cast<size_t>(nre) * 8 * (E / 8 + 4), static_cast<size_t>(a.rd_max) * K) * 4);
  // reductions, flags, sel / wt / weights, probabilities and logits (one per expert the kernel can rank), slot tables
  a.off_misc = take(NW * 8 + 16 + 3 * 32 * 4 + 2 * (DECODE_THREADS / 4) * 4 + (DECODE_MAX_K + 4) * 4 + 4 * DECODE_MAX_K * 4);
  a.off_terms = take(static_cast<size_t>(a.rd_max) * K * nbd * 4);
  a.off_hq = take(static_cast<size_t>(K) * FF + 2 * (static_cast<size_t>(K) * FF / 16) + 4 * (static_cast<size_t>(K) * FF / 256));
  a.off_xr = take(static_cast<size_t>(a.rd_max) * 4);
  a.off_slots = static_cast<uint32_t>(al(o, 128));
  const size_t total = a.off_slots + static_cast<size_t>(K) * a.slot_bytes + 16;
  if (total > static_cast<size_t>(max_smem)) return 1;
  a.smem_bytes = static_cast<uint32_t>(total);
  return 0;
}

// The plan for a context's device; 0 when it fits (else the batched kernels take T = 1 too).
static int plan_decode(const clb200_ctx *c, const clb200_moe_layer &L, DecodeArgs &a) {
  return plan_decode_shape(c->sms, c->max_smem, L, a);
}

int validate(const clb200_moe_layer *L, char *err, size_t errlen) {
  if (!L) { errf(err, errlen, "no layer"); return 1; }
  const int E = L->n_embd, FF = L->n_ff_exp;
  if (E < 256 || E % 256 || E > 4096 || FF < 256 || FF % 256 || FF > 4096) {
    errf(err, errlen, "embedding width %d and expert width %d must be multiples of 256 between 256 and 4096", E, FF);
    return 1;
  }
  if (L->n_expert < 1 || L->n_expert > DECODE_MAX_NE || L->n_used < 1 || L->n_used > DECODE_MAX_K || L->n_used > L->n_expert) {
    errf(err, errlen, "unsupported expert counts (%d experts, %d used; at most %d and %d)", L->n_expert, L->n_used, DECODE_MAX_NE, DECODE_MAX_K);
    return 1;
  }
  if (!expert_type(L->gate.type) || !expert_type(L->up.type) || !expert_type(L->down.type)) {
    errf(err, errlen, "expert tensors are %s / %s / %s; this backend computes Q4_K, Q6_K and Q8_0", type_name(L->gate.type),
         type_name(L->up.type), type_name(L->down.type));
    return 1;
  }
  if (L->gate.type != L->up.type) { errf(err, errlen, "gate (%s) and up (%s) experts must share a type", type_name(L->gate.type), type_name(L->up.type)); return 1; }
  if (L->gate.rows != FF || L->gate.cols != E || L->up.rows != FF || L->up.cols != E || L->down.rows != E || L->down.cols != FF) {
    errf(err, errlen, "expert tensor shapes do not match the widths (%d, %d)", E, FF);
    return 1;
  }
  if (L->gate_slab != FF * row_bytes(L->gate.type, E) || L->up_slab != FF * row_bytes(L->up.type, E) ||
      L->down_slab != E * row_bytes(L->down.type, FF)) {
    errf(err, errlen, "expert slab sizes do not match rows x row bytes");
    return 1;
  }
  if (!L->gate.p || !L->up.p || !L->down.p || !L->router_f || !L->ffn_norm_f) { errf(err, errlen, "a layer tensor is missing"); return 1; }
  return 0;
}

static const char *device_error_text(int code) {
  switch (code) {
    case ERR_WAIT_ROUTER: return "timed out waiting for the router logits of other CTAs (are all CTAs resident?)";
    case ERR_WAIT_EXPERT: return "timed out waiting for an expert's gate/up rows from other CTAs";
    case ERR_WAIT_COPY: return "timed out waiting for a bulk copy into shared memory";
    case ERR_BAD_EXPERT: return "an expert id out of range reached the dispatch";
    case ERR_WAIT_PEER: return "timed out waiting for another GPU's rows or partial sums (does every rank take the same steps?)";
    default: return "unknown device error";
  }
}

// The expert-group kernel (group.cu) on layer L and x (device), with the plan g already made.
static int launch_group(clb200_ctx *c, const clb200_moe_layer &L, GroupArgs &g, float *x, int *sel_out, float *wt_out,
                        cudaStream_t st, char *err, size_t errlen, float *x_out, int *err_out) {
  if (!c->gbuf) {
    CUDA_OR(cudaMalloc(&c->gbuf, GROUP_BUF_BYTES), "allocating the expert-group exchange buffer");
    c->bytes += GROUP_BUF_BYTES;
    CUDA_OR(cudaMemset(c->gbuf, 0, GROUP_BUF_BYTES), "clearing the expert-group exchange buffer");
  }
  if (group_buffer_bytes(c->sms, L.n_embd, L.n_ff_exp, L.n_expert, L.n_used) > GROUP_BUF_BYTES) {
    errf(err, errlen, "the expert-group exchange buffer is too small for this layer");
    return 1;
  }
  g.x_in = x; g.x_out = x_out ? x_out : x;
  g.err_out = err_out;
  g.norm = L.ffn_norm_f; g.router = L.router_f;
  g.gate = L.gate.p; g.up = L.up.p; g.down = L.down.p;
  g.gate_slab = L.gate_slab; g.up_slab = L.up_slab; g.down_slab = L.down_slab;
  g.E = L.n_embd; g.FF = L.n_ff_exp; g.NE = L.n_expert; g.K = L.n_used; g.norm_topk = L.norm_topk;
  g.resid_scale = L.resid_scale; g.eps = L.rms_eps;
  group_set_buffer(g, c->gbuf, c->sms);   // after the shape: the layout follows NE, K, FF and E
  g.err = c->small;
  g.sel_out = sel_out; g.wt_out = wt_out;
  g.force_miss = c->force_miss;
  g.trace = c->trace;
  if (!c->group_attrs_set) {
    CUDA_OR(group_allow_smem(c->max_smem), "kernel attribute");
    c->group_attrs_set = true;
  }
  const GroupFn fn = group_kernel_for(L.gate.type, L.down.type);
  if (reinterpret_cast<const void *>(fn) != c->gocc_fn || g.smem_bytes != c->gocc_smem) {   // once per kernel and size
    int occ = 0;
    CUDA_OR(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, GROUP_THREADS, g.smem_bytes), "occupancy");
    if (occ < 1) { errf(err, errlen, "the expert-group kernel does not fit on an SM (%u bytes of shared memory)", g.smem_bytes); return 1; }
    c->gocc_fn = reinterpret_cast<const void *>(fn);
    c->gocc_smem = g.smem_bytes;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(c->sms);
  cfg.blockDim = dim3(GROUP_THREADS);
  cfg.dynamicSmemBytes = g.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];   // cooperative: every CTA resident at once (they wait on one another), or no launch
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = c->cooperative ? 2 : 1;
  CUDA_OR(cudaLaunchKernelEx(&cfg, fn, g), "launching the expert-group kernel");
  return 0;
}

// The one-token kernel's arguments for layer L (device pointers) in `mode`: plan, scratch, outputs and options (the
// mode-specific inputs are the caller's).
static int decode_args(clb200_ctx *c, const clb200_moe_layer &L, const float *x, int mode, int *sel_out, float *wt_out,
                       float *x_out, int *err_out, DecodeArgs &a, char *err, size_t errlen) {
  const int E = L.n_embd, FF = L.n_ff_exp, NE = L.n_expert, K = L.n_used;
  if (plan_decode(c, L, a)) { errf(err, errlen, "the one-token kernel does not take this layer (K-quant experts only)"); return 1; }
  const Scratch s = plan_scratch(1, E, FF, NE, K, false);
  if (ensure_scratch(c, s.total, err, errlen)) return 1;
  uint8_t *sc = c->scratch;
  a.x_in = x; a.x_out = x_out ? x_out : const_cast<float *>(x);
  a.err_out = err_out;
  a.norm = L.ffn_norm_f; a.router = L.router_f;
  a.gate = L.gate.p; a.up = L.up.p; a.down = L.down.p;
  a.gate_slab = L.gate_slab; a.up_slab = L.up_slab; a.down_slab = L.down_slab;
  a.gate_type = L.gate.type; a.up_type = L.up.type; a.down_type = L.down.type;
  a.E = E; a.FF = FF; a.NE = NE; a.K = K; a.norm_topk = L.norm_topk;
  a.resid_scale = L.resid_scale; a.eps = L.rms_eps;
  a.logits = reinterpret_cast<float *>(sc + s.off_logits);
  a.hg = reinterpret_cast<float *>(sc + s.off_hg);
  a.sel_out = sel_out; a.wt_out = wt_out;
  a.sync = reinterpret_cast<uint32_t *>(c->small + 64);
  a.err = c->small;
  a.trace = c->trace;
  a.mode = mode;
  a.stall_wait = mode == 0 ? c->stall_wait : 0u;
  a.force_miss = mode == 0 ? c->force_miss : 0;
  return 0;
}

int launch_one(clb200_ctx *c, const clb200_moe_layer &L, float *x, int mode, const int *sel_in, const float *wt_in,
               const uint8_t *const *slabs, int *sel_out, float *wt_out, cudaStream_t st, char *err, size_t errlen,
               const SmartRoute *smart, float *x_out, int *err_out, const AheadRoute *ahead) {
  const int E = L.n_embd, FF = L.n_ff_exp, NE = L.n_expert, K = L.n_used;
  if (mode == 0 && !smart && c->decode_kernel == 0 && !c->stall_wait) {
    GroupArgs g{};
    if (plan_group_shape(c->sms, c->max_smem, E, FF, NE, K, L.gate.type, L.up.type, L.down.type, g) == 0) {
      c->signals_done = false;   // its error word reaches err_out only on a failure
      return launch_group(c, L, g, x, sel_out, wt_out, st, err, errlen, x_out, err_out);
    }
  }
  c->signals_done = err_out != nullptr;
  DecodeArgs a{};
  if (decode_args(c, L, x, mode, sel_out, wt_out, x_out, err_out, a, err, errlen)) return 1;
  if (mode == 1 && smart) {
    if (NE > ROUTE_SMEM_MAX_NE || static_cast<size_t>(NE) * 13 + 64 > static_cast<size_t>(K) * a.slot_bytes) {
      errf(err, errlen, "SMART-ROUTE in the one-token kernel takes at most %d experts", ROUTE_SMEM_MAX_NE);
      return 1;
    }
    a.resident = smart->resident;
    a.smart_J = smart->J;
    a.smart_M = smart->M;
    a.smart_tau = smart->tau;
    a.smart_stats = smart->stats;
  }
  if (mode == 1 && ahead && ahead->n > 0) {   // the next layer's rows, products and logits must fit in the free expert slots
    const size_t nre = static_cast<size_t>((NE + c->sms - 1) / c->sms);
    const size_t need = (static_cast<size_t>(E) + nre * E + nre * 8 * (E / 8 + 4) + static_cast<size_t>(NE)) * 4;
    if (need > static_cast<size_t>(K) * a.slot_bytes || ahead->n > NE) {
      errf(err, errlen, "router-ahead does not fit this layer's one-token plan (%zu bytes, %d experts)", need, ahead->n);
      return 1;
    }
    a.ahead_norm = ahead->norm;
    a.ahead_router = ahead->router;
    a.ahead_n = ahead->n;
    a.ahead_out = ahead->out;
  }
  if (mode == 2)
    for (int k = 0; k < K; ++k) {
      a.sel_in[k] = sel_in[k];
      a.wt_in[k] = wt_in[k];
      a.slab[k] = slabs ? slabs[k] : nullptr;
    }
  if (!c->attrs_set) {
    CUDA_OR(decode_allow_smem(c->max_smem), "kernel attribute");
    c->attrs_set = true;
  }
  const DecodeFn fn = decode_kernel_for(a.gate_type, a.down_type);
  if (reinterpret_cast<const void *>(fn) != c->occ_fn || a.smem_bytes != c->occ_smem) {   // checked once per kernel and size
    int occ = 0;
    CUDA_OR(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, DECODE_THREADS, a.smem_bytes), "occupancy");
    if (occ < 1) { errf(err, errlen, "the one-token kernel does not fit on an SM (%u bytes of shared memory)", a.smem_bytes); return 1; }
    c->occ_fn = reinterpret_cast<const void *>(fn);
    c->occ_smem = a.smem_bytes;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(c->sms);
  cfg.blockDim = dim3(DECODE_THREADS);
  cfg.dynamicSmemBytes = a.smem_bytes;
  cfg.stream = st;
  // cooperative: the driver guarantees that every CTA is resident at once (the kernel's CTAs wait on one another), or
  // refuses the launch; programmatic dependent launch lets its prologue overlap the previous kernel's tail
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = c->cooperative ? 2 : 1;
  CUDA_OR(cudaLaunchKernelEx(&cfg, fn, a), "launching the one-token kernel");
  return 0;
}

}  // namespace clb

extern "C" {

clb200_ctx *clb200_open(int device, char *err, size_t errlen) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) { errf(err, errlen, "no CUDA device: %s", e != cudaSuccess ? cudaGetErrorString(e) : "none found"); return nullptr; }
  if (device < 0) cudaGetDevice(&device);
  if (device >= n) { errf(err, errlen, "CUDA device %d does not exist (%d found)", device, n); return nullptr; }
  if (cudaSetDevice(device) != cudaSuccess) { errf(err, errlen, "cannot use CUDA device %d", device); return nullptr; }
  cudaDeviceProp p{};
  cudaGetDeviceProperties(&p, device);
  if (p.major < 10) { errf(err, errlen, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, p.major, p.minor); return nullptr; }
  auto *c = new clb200_ctx();
  c->device = device;
  c->sms = p.multiProcessorCount;
  c->max_smem = static_cast<int>(p.sharedMemPerBlockOptin);
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->small, 4096) != cudaSuccess || cudaMemset(c->small, 0, 4096) != cudaSuccess) {
    errf(err, errlen, "cannot set up a stream and 4 KB on device %d", device);
    clb200_close(c);
    return nullptr;
  }
  c->bytes = 4096;
  return c;
}

void clb200_close(clb200_ctx *c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (auto &l : c->layers) {
    if (l.block) cudaFree(l.block);
    if (l.host_graph) cudaGraphExecDestroy(l.host_graph);
  }
  if (c->scratch) cudaFree(c->scratch);
  if (c->small) cudaFree(c->small);
  if (c->route_buf) cudaFree(c->route_buf);
  if (c->gbuf) cudaFree(c->gbuf);
  if (c->hstage) cudaFreeHost(c->hstage);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

uint64_t clb200_device_bytes(const clb200_ctx *c) { return c ? c->bytes : 0; }

void clb200_set_exact(clb200_ctx *c, int on) {
  if (c) c->exact = on != 0;
}

int clb200_set_option(clb200_ctx *c, int option, int value) {
  if (!c) return 1;
  switch (option) {
    case CLB200_OPT_DECODE_KERNEL: if (value < 0 || value > 1) return 1; c->decode_kernel = value; ++c->graph_gen; return 0;
    case CLB200_OPT_TEST_SPECULATION_MISS: c->force_miss = value != 0; ++c->graph_gen; return 0;
    case CLB200_OPT_TEST_STALL_WAIT: if (value < 0) return 1; c->stall_wait = static_cast<uint32_t>(value); ++c->graph_gen; return 0;
    case CLB200_OPT_COOPERATIVE: c->cooperative = value != 0; ++c->graph_gen; return 0;
    default: return 1;
  }
}

void clb200_set_trace(clb200_ctx *c, void *dev_buf) {
  if (!c) return;
  c->trace = static_cast<unsigned long long *>(dev_buf);
  ++c->graph_gen;
}

int clb200_layer_bind(clb200_ctx *c, const clb200_moe_layer *L, int on_device, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return -1; }
  if (validate(L, err, errlen)) return -1;
  cudaSetDevice(c->device);
  DevLayer dl;
  dl.d = *L;
  const size_t E = L->n_embd, NE = L->n_expert;
  if (!on_device) {
    const size_t sz[5] = {E * 4, NE * E * 4, NE * L->gate_slab, NE * L->up_slab, NE * L->down_slab};
    size_t off[5], tot = 0;
    for (int i = 0; i < 5; ++i) { off[i] = tot; tot = al(tot + sz[i] + 64); }
    if (cudaMalloc(&dl.block, tot) != cudaSuccess) { errf(err, errlen, "cannot allocate %zu bytes for the layer", tot); return -1; }
    uint8_t *b = static_cast<uint8_t *>(dl.block);
    const void *src[5] = {L->ffn_norm_f, L->router_f, L->gate.p, L->up.p, L->down.p};
    for (int i = 0; i < 5; ++i)
      if (cudaMemcpy(b + off[i], src[i], sz[i], cudaMemcpyHostToDevice) != cudaSuccess) {
        errf(err, errlen, "uploading the layer failed");
        cudaFree(dl.block);
        return -1;
      }
    dl.d.ffn_norm_f = reinterpret_cast<const float *>(b + off[0]);
    dl.d.router_f = reinterpret_cast<const float *>(b + off[1]);
    dl.d.gate.p = b + off[2];
    dl.d.up.p = b + off[3];
    dl.d.down.p = b + off[4];
    dl.bytes = tot;
    for (int i = 0; i < 5; ++i) dl.hkey[i] = src[i];
    dl.fp = fingerprint(L);
    c->bytes += tot;
  } else {
    const void *ptrs[5] = {L->ffn_norm_f, L->router_f, L->gate.p, L->up.p, L->down.p};
    for (int i = 0; i < 5; ++i) {
      cudaPointerAttributes at{};
      if (cudaPointerGetAttributes(&at, ptrs[i]) != cudaSuccess || at.type != cudaMemoryTypeDevice || at.device != c->device) {
        cudaGetLastError();
        errf(err, errlen, "layer tensor %d is not memory of device %d", i, c->device);
        return -1;
      }
    }
  }
  dl.live = true;
  c->layers.push_back(dl);
  const int h = static_cast<int>(c->layers.size()) - 1;
  if (!on_device) c->by_gate[L->gate.p] = h;
  return h;
}

int clb200_layer_release(clb200_ctx *c, int layer) {
  if (!c || layer < 0 || layer >= static_cast<int>(c->layers.size()) || !c->layers[layer].live) return 1;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  DevLayer &dl = c->layers[layer];
  auto it = c->by_gate.find(dl.hkey[2]);
  if (it != c->by_gate.end() && it->second == layer) c->by_gate.erase(it);
  if (dl.block) { cudaFree(dl.block); c->bytes -= dl.bytes; }
  if (dl.host_graph) cudaGraphExecDestroy(dl.host_graph);
  dl = DevLayer();
  return 0;
}


// The batched kernels' arguments for layer L (device pointers), T tokens at x, the context's scratch laid out as s.
static BatchArgs batch_args(clb200_ctx *c, const clb200_moe_layer &L, float *x, int T, const Scratch &s, int *sel, float *wt) {
  const int E = L.n_embd, FF = L.n_ff_exp, NE = L.n_expert, K = L.n_used;
  uint8_t *sc = c->scratch;
  BatchArgs b{};
  b.x_in = x; b.x_out = x;
  b.norm = L.ffn_norm_f; b.router = L.router_f;
  b.gate = L.gate.p; b.up = L.up.p; b.down = L.down.p;
  b.gate_slab = L.gate_slab; b.up_slab = L.up_slab; b.down_slab = L.down_slab;
  b.gate_type = L.gate.type; b.up_type = L.up.type; b.down_type = L.down.type;
  b.T = T; b.E = E; b.FF = FF; b.NE = NE; b.K = K; b.norm_topk = L.norm_topk;
  b.resid_scale = L.resid_scale; b.eps = L.rms_eps;
  b.grb = static_cast<uint32_t>(row_bytes(L.gate.type, E));
  b.drb = static_cast<uint32_t>(row_bytes(L.down.type, FF));
  b.xn = reinterpret_cast<float *>(sc + s.off_xn);
  b.xq_qs = reinterpret_cast<int8_t *>(sc + s.off_xq_qs);
  b.xq_d = reinterpret_cast<float *>(sc + s.off_xq_d);
  b.xq_bs = reinterpret_cast<int16_t *>(sc + s.off_xq_bs);
  b.logits = reinterpret_cast<float *>(sc + s.off_logits);
  b.sel = reinterpret_cast<int *>(sc + s.off_bsel);
  b.wt = reinterpret_cast<float *>(sc + s.off_bwt);
  b.counts = reinterpret_cast<int *>(sc + s.off_counts);
  b.offsets = reinterpret_cast<int *>(sc + s.off_offsets);
  b.first = reinterpret_cast<int *>(sc + s.off_first);
  b.todo = reinterpret_cast<int *>(sc + s.off_todo);
  b.pos_token = reinterpret_cast<int *>(sc + s.off_pos_token);
  b.pos_wt = reinterpret_cast<float *>(sc + s.off_pos_wt);
  b.slot_pos = reinterpret_cast<int *>(sc + s.off_slot_pos);
  b.hg = reinterpret_cast<float *>(sc + s.off_bhg);
  b.hq_qs = reinterpret_cast<int8_t *>(sc + s.off_hq_qs);
  b.hq_d = reinterpret_cast<float *>(sc + s.off_hq_d);
  b.hq_bs = reinterpret_cast<int16_t *>(sc + s.off_hq_bs);
  b.hd = reinterpret_cast<float *>(sc + s.off_hd);
  b.sel_out = sel; b.wt_out = wt;
  b.err = c->small;
  // tensor-core expert products where the types allow (Q8_0 down needs the hg planes a tensor-core gate/up writes)
  const bool tcg = !c->exact && L.gate.type == L.up.type && tc_type_supported(L.gate.type, L.gate.p, E, FF) &&
                   tc_type_supported(L.up.type, L.up.p, E, FF);
  const bool tcd = !c->exact && tc_type_supported(L.down.type, L.down.p, E, FF) && (L.down.type != T_Q8_0 || (tcg && L.gate.type == T_Q8_0));
  if (tcg || tcd) b.rs = reinterpret_cast<float *>(sc + s.off_rs);
  if (tcg) {
    b.tc_gu = 1;
    if (L.gate.type == T_Q8_0) {   // xn's fp16 planes (the route kernel writes them)
      b.xh = reinterpret_cast<__half *>(sc + s.off_xh);
      b.xl = reinterpret_cast<__half *>(sc + s.off_xl);
    }
    b.xdh = reinterpret_cast<__half *>(sc + s.off_xdh);
    b.xdl = reinterpret_cast<__half *>(sc + s.off_xdl);
  }
  if (tcd) {
    b.tc_dn = 1;
    b.hgh = reinterpret_cast<__half *>(sc + s.off_hgh);
    b.hgl = reinterpret_cast<__half *>(sc + s.off_hgl);
  }
  return b;
}

// Launches the MoE block for T tokens on device data.
static int run_block(clb200_ctx *c, const DevLayer &dl, float *x, int T, int *sel, float *wt, cudaStream_t st, char *err,
                     size_t errlen) {
  const clb200_moe_layer &L = dl.d;
  const int E = L.n_embd, FF = L.n_ff_exp, NE = L.n_expert, K = L.n_used;
  DecodeArgs probe{};
  if (T == 1 && plan_decode(c, L, probe) == 0) return launch_one(c, L, x, 0, nullptr, nullptr, nullptr, sel, wt, st, err, errlen);
  const Scratch s = plan_scratch(T, E, FF, NE, K, true);
  if (ensure_scratch(c, s.total, err, errlen)) return 1;
  BatchArgs b = batch_args(c, L, x, T, s, sel, wt);
  const int rc = launch_batched(b, st);
  if (rc) { errf(err, errlen, "launching the batched kernels: %s", cudaGetErrorString(static_cast<cudaError_t>(rc))); return 1; }
  return 0;
}

int clb200_moe_ffn_dev(clb200_ctx *c, int layer, float *x, int T, int *sel, float *wt, void *stream, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (layer < 0 || layer >= static_cast<int>(c->layers.size()) || !c->layers[layer].live) { errf(err, errlen, "no layer %d", layer); return 1; }
  if (T < 1 || T > 512) { errf(err, errlen, "%d tokens: a call takes 1 to 512", T); return 1; }
  if (!x) { errf(err, errlen, "no activations"); return 1; }
  cudaSetDevice(c->device);
  return run_block(c, c->layers[layer], x, T, sel, wt, stream ? static_cast<cudaStream_t>(stream) : c->stream, err, errlen);
}

static const DevLayer *ep_layer(clb200_ctx *c, int layer, int T, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return nullptr; }
  if (layer < 0 || layer >= static_cast<int>(c->layers.size()) || !c->layers[layer].live) { errf(err, errlen, "no layer %d", layer); return nullptr; }
  if (T < 1 || T > 32768) { errf(err, errlen, "%d tokens: an expert-parallel call takes 1 to 32768", T); return nullptr; }
  const clb200_moe_layer &L = c->layers[layer].d;
  if (L.gate.type == T_Q8_0) { errf(err, errlen, "expert-parallel calls take K-quant gate/up experts (Q4_K, Q6_K)"); return nullptr; }
  cudaSetDevice(c->device);
  return &c->layers[layer];
}

int clb200_ep_route(clb200_ctx *c, int layer, float *x, int T, int *sel, float *wt, int8_t *xq_qs, float *xq_d, int16_t *xq_bs,
                    void *stream, char *err, size_t errlen) {
  const DevLayer *dl = ep_layer(c, layer, T, err, errlen);
  if (!dl) return 1;
  if (!x || !sel || !wt || !xq_qs || !xq_d || !xq_bs) { errf(err, errlen, "a buffer is missing"); return 1; }
  const clb200_moe_layer &L = dl->d;
  const Scratch s = plan_scratch(T, L.n_embd, L.n_ff_exp, L.n_expert, L.n_used, true);
  if (ensure_scratch(c, s.total, err, errlen)) return 1;
  BatchArgs b = batch_args(c, L, x, T, s, nullptr, nullptr);
  b.sel = sel; b.wt = wt;
  b.xq_qs = xq_qs; b.xq_d = xq_d; b.xq_bs = xq_bs;
  const int rc = launch_route(b, stream ? static_cast<cudaStream_t>(stream) : c->stream);
  if (rc) { errf(err, errlen, "launching the router: %s", cudaGetErrorString(static_cast<cudaError_t>(rc))); return 1; }
  return 0;
}

int clb200_ep_experts(clb200_ctx *c, int layer, int T, const int8_t *xq_qs, const float *xq_d, const int16_t *xq_bs, const int *sel,
                      const float *wt, float *partial, void *stream, char *err, size_t errlen) {
  const DevLayer *dl = ep_layer(c, layer, T, err, errlen);
  if (!dl) return 1;
  if (!partial || !sel || !wt || !xq_qs || !xq_d || !xq_bs) { errf(err, errlen, "a buffer is missing"); return 1; }
  const clb200_moe_layer &L = dl->d;
  const Scratch s = plan_scratch(T, L.n_embd, L.n_ff_exp, L.n_expert, L.n_used, true);
  if (ensure_scratch(c, s.total, err, errlen)) return 1;
  BatchArgs b = batch_args(c, L, partial, T, s, nullptr, nullptr);
  b.x_in = nullptr;
  b.x_out = partial;
  b.ep = 1;
  b.sel = const_cast<int *>(sel);
  b.wt = const_cast<float *>(wt);
  b.xq_qs = const_cast<int8_t *>(xq_qs);
  b.xq_d = const_cast<float *>(xq_d);
  b.xq_bs = const_cast<int16_t *>(xq_bs);
  const int rc = launch_experts(b, stream ? static_cast<cudaStream_t>(stream) : c->stream);
  if (rc) { errf(err, errlen, "launching the expert kernels: %s", cudaGetErrorString(static_cast<cudaError_t>(rc))); return 1; }
  return 0;
}

int clb200_moe_dispatch(clb200_ctx *c, int T, int n_expert, int n_used, const int *sel, const float *wt, int *todo, int *offsets,
                        int *pos_token, float *pos_wt, void *stream, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (T < 1 || T > 32768 || n_expert < 1 || n_expert > DECODE_MAX_NE || n_used < 1 || n_used > DECODE_MAX_K || n_used > n_expert) {
    errf(err, errlen, "dispatch of %d tokens, %d experts, %d used: takes 1 to 32768 tokens, at most %d experts and %d used", T,
         n_expert, n_used, DECODE_MAX_NE, DECODE_MAX_K);
    return 1;
  }
  if (!sel || !wt || !todo || !offsets || !pos_token || !pos_wt) { errf(err, errlen, "a buffer is missing"); return 1; }
  cudaSetDevice(c->device);
  const size_t TK = static_cast<size_t>(T) * n_used, o_first = al(static_cast<size_t>(n_expert) * 4),
               o_slot = o_first + al(static_cast<size_t>(n_expert) * 4);
  if (ensure_scratch(c, o_slot + al(TK * 4), err, errlen)) return 1;
  BatchArgs b{};
  b.T = T; b.NE = n_expert; b.K = n_used;
  b.sel = const_cast<int *>(sel);
  b.wt = const_cast<float *>(wt);
  b.counts = reinterpret_cast<int *>(c->scratch);
  b.first = reinterpret_cast<int *>(c->scratch + o_first);
  b.slot_pos = reinterpret_cast<int *>(c->scratch + o_slot);
  b.offsets = offsets; b.todo = todo; b.pos_token = pos_token; b.pos_wt = pos_wt;
  b.err = c->small;
  const int rc = launch_dispatch(b, stream ? static_cast<cudaStream_t>(stream) : c->stream);
  if (rc) { errf(err, errlen, "launching the dispatch: %s", cudaGetErrorString(static_cast<cudaError_t>(rc))); return 1; }
  return 0;
}

// 1 with err set when the device error word read back is non-zero; the word and the counters a failed kernel may have left
// behind are cleared.
static int report_device_error(clb200_ctx *c, int code, char *err, size_t errlen) {
  if (!code) return 0;
  errf(err, errlen, "device error %d: %s", code, device_error_text(code));
  cudaMemset(c->small, 0, 4096);
  if (c->gbuf) cudaMemset(c->gbuf, 0, GROUP_BUF_BYTES);   // a failed launch may leave words the next one could take as its own
  return 1;
}

int clb200_status(clb200_ctx *c, char *err, size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  cudaSetDevice(c->device);
  CUDA_OR(cudaDeviceSynchronize(), "device");
  int code = 0;
  CUDA_OR(cudaMemcpy(&code, c->small, 4, cudaMemcpyDeviceToHost), "reading the device error word");
  return report_device_error(c, code, err, errlen);
}

// One token of a host call through the one-token kernel, with no copy-engine transfer: x is copied into the mapped pinned
// staging on the host and read from there by a small kernel; the one-token kernel writes x, sel and wt into the staging
// and its last CTA the error word; one wait on the stream. (Each copy-engine transfer costs several microseconds of
// latency, as much as a quarter of the kernel at one token.)
static int host_call_one(clb200_ctx *c, DevLayer &dl, float *x, int *sel_out, float *wt_out, char *err, size_t errlen) {
  const clb200_moe_layer &L = dl.d;
  const int E = L.n_embd, K = L.n_used;
  const size_t xb = static_cast<size_t>(E) * 4, kb = static_cast<size_t>(K) * 4;
  const size_t o_out = al(xb), o_sel = o_out + al(xb), o_wt = o_sel + al(kb), o_err = o_wt + al(kb);
  if (ensure_hstage(c, o_err + 256, err, errlen)) return 1;
  const Scratch s = plan_scratch(1, E, L.n_ff_exp, L.n_expert, K, false);
  if (ensure_scratch(c, s.total, err, errlen)) return 1;
  float *dx = reinterpret_cast<float *>(c->scratch + s.off_x);
  uint8_t *h = c->hstage, *hd = c->hstage_dev;
  volatile int *herr = reinterpret_cast<volatile int *>(h + o_err);
  constexpr int PENDING = -1;   // device error codes are >= 0
  *herr = PENDING;
  std::memcpy(h, x, xb);
  // Every argument of the two launches is fixed for a layer (x goes through the staging), so from the layer's second call
  // on they are one graph launch: the first call sets the kernels' attributes and the exchange buffers up eagerly.
  if (dl.host_graph && dl.host_graph_gen != c->graph_gen) {
    cudaGraphExecDestroy(dl.host_graph);
    dl.host_graph = nullptr;
  }
  auto launches = [&]() -> int {
    CUDA_OR(launch_stage_in(reinterpret_cast<const float *>(hd), dx, E, c->stream), "staging x");
    return launch_one(c, L, dx, 0, nullptr, nullptr, nullptr, reinterpret_cast<int *>(hd + o_sel), reinterpret_cast<float *>(hd + o_wt),
                      c->stream, err, errlen, nullptr, reinterpret_cast<float *>(hd + o_out), reinterpret_cast<int *>(hd + o_err));
  };
  if (!dl.host_graph && dl.host_calls >= 1) {
    cudaGraph_t g = nullptr;
    CUDA_OR(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "capturing the host call");
    const int rc = launches();
    const cudaError_t ec = cudaStreamEndCapture(c->stream, &g);
    if (rc || ec != cudaSuccess || cudaGraphInstantiate(&dl.host_graph, g, 0) != cudaSuccess) {
      dl.host_graph = nullptr;
      cudaGetLastError();   // a failed capture leaves no sticky error; this call runs its launches directly below
    } else {
      dl.host_graph_gen = c->graph_gen;
    }
    if (g) cudaGraphDestroy(g);
  }
  ++dl.host_calls;
  if (dl.host_graph) {
    CUDA_OR(cudaGraphLaunch(dl.host_graph, c->stream), "launching the host call's graph");
  } else if (launches()) {
    cudaStreamSynchronize(c->stream);   // the staging kernel may still read the staging, which the next call rewrites
    return 1;
  }
  int code = PENDING;
  if (c->signals_done) {
    // The grid-wide kernel's last CTA writes the error word into the mapped staging after a system-wide fence, so the
    // results are in host memory once it arrives: spin on it, and ask the stream now and then (a launch that failed writes
    // nothing), instead of a blocking synchronisation.
    for (uint32_t n = 1;; ++n) {
      code = *herr;
      if (code != PENDING) break;
      if ((n & 4095) == 0 && cudaStreamQuery(c->stream) != cudaErrorNotReady) {
        code = *herr;
        break;
      }
    }
  }
  if (code == PENDING) {
    CUDA_OR(cudaStreamSynchronize(c->stream), "running the MoE block");
    code = *herr;
    if (code == PENDING) code = 0;   // a kernel that reports its error word only on a failure
  }
  if (report_device_error(c, code, err, errlen)) return 1;
  std::memcpy(x, h + o_out, xb);
  if (sel_out) std::memcpy(sel_out, h + o_sel, kb);
  if (wt_out) std::memcpy(wt_out, h + o_wt, kb);
  return 0;
}

int clb200_moe_ffn(clb200_ctx *c, const clb200_moe_layer *L, float *x, int T, int *sel_out, float *wt_out, char *err,
                   size_t errlen) {
  if (!c) { errf(err, errlen, "no context"); return 1; }
  if (T < 1 || T > 512) { errf(err, errlen, "%d tokens: a call takes 1 to 512", T); return 1; }
  if (!x || !L) { errf(err, errlen, "no activations or no layer"); return 1; }
  cudaSetDevice(c->device);
  int h = -1;
  auto it = c->by_gate.find(L->gate.p);
  if (it != c->by_gate.end()) {
    const DevLayer &dl = c->layers[it->second];
    if (dl.hkey[0] == L->ffn_norm_f && dl.hkey[1] == L->router_f && dl.hkey[3] == L->up.p && dl.hkey[4] == L->down.p &&
        dl.fp == fingerprint(L))   // the shape fields are inside the fingerprint; the layer was validated when it was bound
      h = it->second;
    else
      clb200_layer_release(c, it->second);   // the host memory now holds something else: drop the stale upload
  }
  if (h < 0) {
    h = clb200_layer_bind(c, L, 0, err, errlen);
    if (h < 0) return 1;
  }
  DevLayer &dl = c->layers[h];
  dl.d.resid_scale = L->resid_scale;   // the scalars the fingerprint leaves out follow the caller's struct
  dl.d.rms_eps = L->rms_eps;
  DecodeArgs probe{};
  if (T == 1 && plan_decode(c, dl.d, probe) == 0) return host_call_one(c, dl, x, sel_out, wt_out, err, errlen);
  const int E = L->n_embd, K = L->n_used;
  const Scratch s = plan_scratch(T, E, L->n_ff_exp, L->n_expert, K, true);   // the staging buffers lead either plan
  if (ensure_scratch(c, s.total, err, errlen)) return 1;
  float *dx = reinterpret_cast<float *>(c->scratch + s.off_x);
  int *dsel = reinterpret_cast<int *>(c->scratch + s.off_sel);
  float *dwt = reinterpret_cast<float *>(c->scratch + s.off_wt);
  const size_t xb = static_cast<size_t>(T) * E * 4, kb = static_cast<size_t>(T) * K * 4;
  // The results come back through pinned staging: x (up to 1 MB; larger x goes straight to the caller's buffer), sel and wt,
  // which lie in that order at the start of scratch, as one copy, and the error word as a second; then one wait on the
  // stream. A copy per buffer and a device-wide synchronisation to read the error word cost more than the kernel at T = 1.
  const bool stage_x = xb <= (size_t(1) << 20);
  const size_t lo = stage_x ? s.off_x : s.off_sel, span = s.off_wt + kb - lo, at_err = al(span, 16);
  if (ensure_hstage(c, at_err + 16, err, errlen)) return 1;
  CUDA_OR(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, c->stream), "copying x to the device");
  if (run_block(c, dl, dx, T, dsel, dwt, c->stream, err, errlen)) return 1;
  if (!stage_x) CUDA_OR(cudaMemcpyAsync(x, dx, xb, cudaMemcpyDeviceToHost, c->stream), "copying x back");
  CUDA_OR(cudaMemcpyAsync(c->hstage, c->scratch + lo, span, cudaMemcpyDeviceToHost, c->stream), "copying the results back");
  CUDA_OR(cudaMemcpyAsync(c->hstage + at_err, c->small, 4, cudaMemcpyDeviceToHost, c->stream), "reading the device error word");
  CUDA_OR(cudaStreamSynchronize(c->stream), "running the MoE block");
  int code = 0;
  std::memcpy(&code, c->hstage + at_err, 4);
  if (report_device_error(c, code, err, errlen)) return 1;
  if (stage_x) std::memcpy(x, c->hstage + (s.off_x - lo), xb);
  if (sel_out) std::memcpy(sel_out, c->hstage + (s.off_sel - lo), kb);
  if (wt_out) std::memcpy(wt_out, c->hstage + (s.off_wt - lo), kb);
  return 0;
}

}  // extern "C"

namespace clb {
int run_moe_block(clb200_ctx *c, const DevLayer &dl, float *x, int T, int *sel, float *wt, cudaStream_t st, char *err,
                  size_t errlen) {
  return run_block(c, dl, x, T, sel, wt, st, err, errlen);
}
}  // namespace clb
