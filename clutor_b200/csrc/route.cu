// SMART-ROUTE entry points: the reference's cl_route (c/src/route.h:26, c/src/route.c:13-52) on the GPU, one CTA per
// token (route_cta in route.cuh). Host code plus one small kernel.
#include <cstring>

#include "ctx.cuh"
#include "route.cuh"

using namespace clb;

namespace {

constexpr int ROUTE_THREADS = 256;

static_assert(sizeof(clb200_route_result) == 152, "clb200_route_result must match cl_route_result");
static_assert(sizeof(clb200_smart) == 24, "clb200_smart must match cl_smart");

// Token t: logits [t * E, (t + 1) * E), residency resident + t * rstride (rstride 0: one set for every token).
__global__ void __launch_bounds__(ROUTE_THREADS) route_kernel(const float *logits, int E, int K, SmartCfg cfg,
                                                               const uint8_t *resident, int rstride, clb200_route_result *out) {
  __shared__ double p[ROUTE_MAX_E];
  __shared__ int order[ROUTE_MAX_E];
  __shared__ uint8_t taken[ROUTE_MAX_E];
  __shared__ double red[ROUTE_THREADS / 32];
  __shared__ int sel[ROUTE_MAX_K];
  __shared__ RouteStats st;
  const int t = blockIdx.x;
  const uint8_t *res = resident ? resident + static_cast<size_t>(t) * rstride : nullptr;
  route_cta(logits + static_cast<size_t>(t) * E, E, K, cfg, res, p, order, taken, red, sel, &st);
  clb200_route_result *o = out + t;
  const int tid = threadIdx.x;
  if (tid < ROUTE_MAX_K) o->selected[tid] = tid < K ? sel[tid] : 0;
  if (tid == 0) {
    o->k = K;
    o->substituted = st.substituted;
    o->dropped_mass = st.dropped_mass;
    o->max_delta = st.max_delta;
  }
}

SmartCfg cfg_of(const clb200_smart *s) {
  SmartCfg c{};
  if (s) {
    c.enabled = s->enabled;
    c.J = s->J;
    c.M = s->M;
    c.tau = s->tau;
  }
  return c;
}

bool args_ok(int E, int K) { return E > 0 && E <= ROUTE_MAX_E && K > 0 && K <= ROUTE_MAX_K && K <= E; }

}  // namespace

namespace clb {
int launch_route_kernel(const float *logits, int T, int E, int K, const clb200_smart *smart, const uint8_t *resident,
                        int rstride, clb200_route_result *out, cudaStream_t st) {
  if (T <= 0) return 0;
  route_kernel<<<T, ROUTE_THREADS, 0, st>>>(logits, E, K, cfg_of(smart), resident, rstride, out);
  return cudaGetLastError() != cudaSuccess;
}
}  // namespace clb

extern "C" {

int clb200_route(clb200_ctx *c, const float *logits, int E, int K, const clb200_smart *smart, const uint8_t *resident,
                 clb200_route_result *out, char *err, size_t errlen) {
  if (!args_ok(E, K)) return -1;   // as cl_route: E, K out of range
  if (!c || !logits || !out) { errf(err, errlen, "no context, logits or result"); return 1; }
  cudaSetDevice(c->device);
  if (!c->route_buf) {
    CUDA_OR(cudaMalloc(&c->route_buf, ROUTE_BUF_BYTES), "allocating the routing buffer");
    c->bytes += ROUTE_BUF_BYTES;
  }
  float *dl = reinterpret_cast<float *>(c->route_buf);
  uint8_t *dr = c->route_buf + ROUTE_MAX_E * 4;
  clb200_route_result *dout = reinterpret_cast<clb200_route_result *>(c->route_buf + ROUTE_MAX_E * 5);
  const bool smart_on = smart && smart->enabled && resident;
  CUDA_OR(cudaMemcpyAsync(dl, logits, static_cast<size_t>(E) * 4, cudaMemcpyHostToDevice, c->stream), "logits upload");
  if (smart_on) CUDA_OR(cudaMemcpyAsync(dr, resident, static_cast<size_t>(E), cudaMemcpyHostToDevice, c->stream), "residency upload");
  if (launch_route_kernel(dl, 1, E, K, smart, smart_on ? dr : nullptr, 0, dout, c->stream)) {
    errf(err, errlen, "launching the routing kernel: %s", cudaGetErrorString(cudaGetLastError()));
    return 1;
  }
  CUDA_OR(cudaMemcpyAsync(out, dout, sizeof(clb200_route_result), cudaMemcpyDeviceToHost, c->stream), "result download");
  CUDA_OR(cudaStreamSynchronize(c->stream), "routing");
  return 0;
}

int clb200_route_dev(clb200_ctx *c, const float *logits, int T, int E, int K, const clb200_smart *smart,
                     const uint8_t *resident, int resident_stride, clb200_route_result *out, void *stream) {
  if (!args_ok(E, K) || T < 0 || resident_stride < 0) return -1;
  if (!c || (T > 0 && (!logits || !out))) return 1;
  cudaSetDevice(c->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  return launch_route_kernel(logits, T, E, K, smart, smart && smart->enabled ? resident : nullptr, resident_stride, out, st);
}

}  // extern "C"
