// The one-token MoE block for callers that cannot allocate device memory.
//
// Some hosts must not call cudaMalloc once they are running: an engine whose device memory is all carved out up front by
// another allocator (a framework's caching pool owns the GPU, and a raw cudaMalloc beside it fails or fragments), or one
// that decodes under a latency budget (cudaMalloc can synchronise the device and take milliseconds). Such a host owns its
// inputs and outputs and cannot give this library a context with scratch. clb200_moe_ffn_decode_noalloc runs the same
// one-token kernel as clb200_moe_ffn_dev with its scratch -- the router logits, the experts' hg rows, three grid counters
// and the error word -- in a fixed array of this file that every device holds from the moment it loads the library.
//
// The array's device address is looked up once per device (on the first call with that device current) and kept for the
// life of the process: after cudaDeviceReset the module is loaded again and the array may move, so this entry point must
// not be used across a device reset.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/clb200.h"
#include "common.cuh"
#include "decode.cuh"

namespace clb {

int plan_decode_shape(int sms, int max_smem, const clb200_moe_layer &L, DecodeArgs &a);   // api.cu
int validate(const clb200_moe_layer *L, char *err, size_t errlen);                           // api.cu

namespace {

// Scratch layout: [0, 4) device error word; [256, 268) the kernel's three counters; [512, 1024) router logits of up to
// 128 experts; [1024, 1024 + 4 * NOALLOC_MAX_HG) hg rows, n_used x n_ff_exp floats.
constexpr size_t NOALLOC_MAX_HG = 16384;
constexpr size_t NOALLOC_BYTES = 1024 + 4 * NOALLOC_MAX_HG;   // 66,560 bytes
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_BYTES];

struct DeviceSetup {
  bool ready = false;
  uint8_t *scratch = nullptr;   // device address of g_noalloc_scratch on this device
  int sms = 0, max_smem = 0;
  const void *occ_fn = nullptr;   // the kernel and shared size last found to fit an SM on this device
  uint32_t occ_smem = 0;
};
std::mutex g_setup_mu;
DeviceSetup g_setup[64];

void errf(char *err, size_t errlen, const char *fmt, ...) {
  if (!err || !errlen) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, errlen, fmt, ap);
  va_end(ap);
}

}  // namespace
}  // namespace clb

using namespace clb;

extern "C" int clb200_moe_ffn_decode_noalloc(const clb200_moe_layer *L, float *x, int *sel_out, float *wt_out, void *stream,
                                              char *err, size_t errlen) {
  if (!L || !x) { errf(err, errlen, "no layer or no activations"); return 1; }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { errf(err, errlen, "no usable current CUDA device"); return 1; }
  DeviceSetup su;
  {
    // once per device, with that device current: the array's device address (the host-side name is only a stand-in)
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup &s = g_setup[dev];
    if (!s.ready) {
      void *ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess) { errf(err, errlen, "cannot locate the scratch array on device %d: %s", dev, cudaGetErrorString(e)); return 1; }
      if (cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&s.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
          decode_allow_smem(s.max_smem) != cudaSuccess) {
        errf(err, errlen, "cannot set up device %d", dev);
        return 1;
      }
      s.scratch = static_cast<uint8_t *>(ptr);
      s.ready = true;
    }
    su = s;
  }
  // the checks of the context path first (widths 256..4096, types, gate/up sharing a type, slab sizes), then this entry
  // point's own limits
  if (validate(L, err, errlen)) return 1;
  const int E = L->n_embd, FF = L->n_ff_exp, NE = L->n_expert, K = L->n_used;
  if (NE < 1 || NE > 128 || K < 1 || K > NE || static_cast<size_t>(K) * FF > NOALLOC_MAX_HG) {
    errf(err, errlen, "%d experts, %d used, expert width %d: the allocation-free entry point takes at most 128 experts and "
         "n_used * n_ff_exp <= %zu (its fixed scratch is %zu bytes)", NE, K, FF, NOALLOC_MAX_HG, NOALLOC_BYTES);
    return 1;
  }
  DecodeArgs a{};
  if (plan_decode_shape(su.sms, su.max_smem, *L, a)) {
    errf(err, errlen, "this layer shape or weight type is not one the one-token kernel takes (K-quant experts, at most 16 used)");
    return 1;
  }
  const DecodeFn fn = decode_kernel_for(L->gate.type, L->down.type);
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);   // checked once per device, kernel and shared size
    DeviceSetup &s = g_setup[dev];
    if (reinterpret_cast<const void *>(fn) != s.occ_fn || a.smem_bytes != s.occ_smem) {
      int occ = 0;
      const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, DECODE_THREADS, a.smem_bytes);
      if (e != cudaSuccess || occ < 1) {
        errf(err, errlen, "the one-token kernel does not fit on an SM of device %d (%u bytes of shared memory)", dev, a.smem_bytes);
        return 1;
      }
      s.occ_fn = reinterpret_cast<const void *>(fn);
      s.occ_smem = a.smem_bytes;
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  a.x_in = x; a.x_out = x;
  a.norm = L->ffn_norm_f; a.router = L->router_f;
  a.gate = L->gate.p; a.up = L->up.p; a.down = L->down.p;
  a.gate_slab = L->gate_slab; a.up_slab = L->up_slab; a.down_slab = L->down_slab;
  a.gate_type = L->gate.type; a.up_type = L->up.type; a.down_type = L->down.type;
  a.E = E; a.FF = FF; a.NE = NE; a.K = K; a.norm_topk = L->norm_topk;
  a.resid_scale = L->resid_scale; a.eps = L->rms_eps;
  a.err = reinterpret_cast<int *>(su.scratch);
  a.sync = reinterpret_cast<uint32_t *>(su.scratch + 256);
  a.logits = reinterpret_cast<float *>(su.scratch + 512);
  a.hg = reinterpret_cast<float *>(su.scratch + 1024);
  a.sel_out = sel_out; a.wt_out = wt_out;
  // the array keeps the last call's contents: the error word and the counters must start at zero
  cudaError_t e = cudaMemsetAsync(su.scratch, 0, 512, st);
  if (e != cudaSuccess) { errf(err, errlen, "clearing the scratch counters: %s", cudaGetErrorString(e)); return 1; }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(su.sms);
  cfg.blockDim = dim3(DECODE_THREADS);
  cfg.dynamicSmemBytes = a.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];   // cooperative: every CTA resident at once (they wait on one another), or no launch
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, fn, a);
  if (e != cudaSuccess) { errf(err, errlen, "launching the one-token kernel: %s", cudaGetErrorString(e)); return 1; }
  // the error word comes back on the caller's stream (a copy on the legacy stream would also wait for other streams' work)
  int code = 0;
  e = cudaMemcpyAsync(&code, su.scratch, sizeof code, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) { errf(err, errlen, "reading the device error word: %s", cudaGetErrorString(e)); return 1; }
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) { errf(err, errlen, "running the one-token kernel: %s", cudaGetErrorString(e)); return 1; }
  if (code) { errf(err, errlen, "device error %d (a bounded wait ran out)", code); return 1; }
  return 0;
}
