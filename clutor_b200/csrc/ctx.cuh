// Internals shared by the host-side translation units (api.cu, store.cu): error formatting, row sizes, the layer and
// context records, and the one-token launch.
#pragma once
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/clb200.h"
#include "common.cuh"
#include "decode.cuh"

namespace clb {

inline void errf(char *err, size_t errlen, const char *fmt, ...) {
  if (!err || !errlen) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, errlen, fmt, ap);
  va_end(ap);
}

inline uint64_t row_bytes(uint32_t t, uint64_t n) {
  switch (t) {
    case T_Q4_K: return n / 256 * 144;
    case T_Q6_K: return n / 256 * 210;
    case T_Q8_0: return n / 32 * 34;
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    default: return 0;
  }
}
inline bool expert_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0; }
inline const char *type_name(uint32_t t) {
  switch (t) {
    case T_Q4_K: return "Q4_K";
    case T_Q6_K: return "Q6_K";
    case T_Q8_0: return "Q8_0";
    case T_F32: return "F32";
    case T_F16: return "F16";
    default: return "an unsupported type";
  }
}
inline size_t al(size_t v, size_t a = 256) { return (v + a - 1) / a * a; }

#define CUDA_OR(call, msg)                                                                                            \
  do {                                                                                                                \
    cudaError_t e_ = (call);                                                                                          \
    if (e_ != cudaSuccess) { errf(err, errlen, "%s: %s", msg, cudaGetErrorString(e_)); return 1; }                    \
  } while (0)

struct DevLayer {
  clb200_moe_layer d{};              // device pointers
  const void *hkey[5] = {};          // host pointers of norm, router, gate, up, down (0 when bound on the device)
  uint64_t fp = 0;                   // fingerprint of the host tensors' shapes and edge bytes (uploaded layers)
  void *block = nullptr;             // the owned device copy (upload), else null
  size_t bytes = 0;
  bool live = false;
  // a host call's launches at one token (stage-in and one-token kernel), as a graph: captured on the layer's second host call
  // and replayed while the context's launch state (graph_gen) is unchanged
  cudaGraphExec_t host_graph = nullptr;
  uint64_t host_graph_gen = 0;
  int host_calls = 0;
};

// FNV-1a over the layer's shape fields and the first and last 16 bytes of each host tensor: a cheap check, made on every
// host call, that a host pointer seen before still holds the weights that were uploaded from it (a freed and reused buffer
// usually does not).
inline uint64_t fingerprint(const clb200_moe_layer *L) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](const void *p, size_t n) {
    const uint8_t *b = static_cast<const uint8_t *>(p);
    for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
  };
  const int shape[9] = {L->n_embd, L->n_ff_exp, L->n_expert, L->n_used, L->norm_topk, static_cast<int>(L->gate.type),
                        static_cast<int>(L->up.type), static_cast<int>(L->down.type), 0};
  mix(shape, sizeof shape);
  const size_t E = L->n_embd, NE = L->n_expert;
  const void *ptr[5] = {L->ffn_norm_f, L->router_f, L->gate.p, L->up.p, L->down.p};
  const size_t sz[5] = {E * 4, NE * E * 4, NE * L->gate_slab, NE * L->up_slab, NE * L->down_slab};
  for (int i = 0; i < 5; ++i) {
    const size_t n = sz[i] < 16 ? sz[i] : 16;
    mix(ptr[i], n);
    mix(static_cast<const uint8_t *>(ptr[i]) + sz[i] - n, n);
  }
  return h;
}

// Validates a layer description (shapes, types, slabs); 0 when the block can run it.
int validate(const clb200_moe_layer *L, char *err, size_t errlen);
// Shared-memory plan of the one-token kernel; 0 when it fits.
int plan_decode_shape(int sms, int max_smem, const clb200_moe_layer &L, DecodeArgs &a);

}  // namespace clb

struct clb200_ctx {
  int device = 0, sms = 0, max_smem = 0;
  cudaStream_t stream = nullptr;
  std::vector<clb::DevLayer> layers;
  std::unordered_map<const void *, int> by_gate;   // host gate pointer -> layer index
  int *small = nullptr;                            // [0] device error word, [64..] counters of the one-token kernel
  uint8_t *scratch = nullptr;
  size_t scratch_cap = 0;
  uint8_t *hstage = nullptr;                       // pinned, mapped host staging of a host call's x, results and error word
  uint8_t *hstage_dev = nullptr;                   // its device address
  size_t hstage_cap = 0;
  const void *occ_fn = nullptr;                    // the one-token kernel and shared size last found to fit an SM
  uint32_t occ_smem = 0;
  uint64_t bytes = 0;
  bool attrs_set = false;
  unsigned long long *trace = nullptr;             // phase trace of the one-token kernel (device, 32 per CTA) or null
  uint8_t *route_buf = nullptr;                    // clb200_route: logits, residency and result on the device
  bool exact = false;                              // batched expert products on the integer path only (no tensor cores)
  uint8_t *gbuf = nullptr;                         // the expert-group kernel's exchange buffer (zeroed once, its alone)
  bool group_attrs_set = false;
  const void *gocc_fn = nullptr;                   // the expert-group kernel and shared size last found to fit an SM
  uint32_t gocc_smem = 0;
  uint64_t graph_gen = 1;                          // bumped whenever a captured host-call graph would go stale (scratch or
                                                   // staging moved, a trace buffer or an option set)
  int decode_kernel = 1;                           // CLB200_OPT_DECODE_KERNEL
  bool signals_done = false;                       // the last one-token launch writes its error word to host memory on exit
  int force_miss = 0;                              // CLB200_OPT_TEST_SPECULATION_MISS
  bool cooperative = true;                         // CLB200_OPT_COOPERATIVE
  uint32_t stall_wait = 0;                         // CLB200_OPT_TEST_STALL_WAIT
};
constexpr size_t GROUP_BUF_BYTES = size_t(4) << 20;   // >= group_buffer_bytes() of every shape the kernel takes
constexpr size_t ROUTE_BUF_BYTES = 1024 * 5 + 256;

namespace clb {
// The one-token kernel on layer L (device pointers) and x [n_embd] (device) in `mode` (DecodeArgs::mode); for mode 2,
// sel_in / wt_in [n_used] (host) and slabs [n_used] (device addresses, or null entries for L's own tensors). Returns 1 with
// err set when the layer does not suit the one-token kernel or the launch fails.
// smart (mode 1 only, may be null): SMART-ROUTE with the residency and settings it holds (DecodeArgs::resident ...).
// x_out (null: x itself) receives the result; err_out (null: none) is DecodeArgs::err_out.
struct SmartRoute {
  const uint8_t *resident;   // device-visible [n_expert] bytes
  int J, M;
  double tau;
  void *stats;               // device-visible RouteStats
};
// Router-ahead for a routing-only launch (c/src/forward.c:937-946): the next layer's norm and router (device), and where
// its top n experts go (device-visible [n]).
struct AheadRoute {
  const float *norm, *router;
  int n;
  int *out;
};
int launch_one(clb200_ctx *c, const clb200_moe_layer &L, float *x, int mode, const int *sel_in, const float *wt_in,
               const uint8_t *const *slabs, int *sel_out, float *wt_out, cudaStream_t st, char *err, size_t errlen,
               const SmartRoute *smart = nullptr, float *x_out = nullptr, int *err_out = nullptr, const AheadRoute *ahead = nullptr);
// The MoE block of layer dl on T tokens of device data x (updated in place), queued on st: the one-token kernel for T = 1,
// the batched kernels otherwise; sel / wt (device, [T * n_used]) may be null.
int run_moe_block(clb200_ctx *c, const DevLayer &dl, float *x, int T, int *sel, float *wt, cudaStream_t st, char *err,
                  size_t errlen);
// The routing kernel of route.cu: T tokens, one CTA each; returns non-zero when the launch fails.
int launch_route_kernel(const float *logits, int T, int E, int K, const clb200_smart *smart, const uint8_t *resident,
                        int rstride, clb200_route_result *out, cudaStream_t st);
}  // namespace clb
