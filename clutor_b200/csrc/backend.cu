// The "b200" cl_backend for the reference's plugin seam, cl_matvec_batch (c/src/quant.c:995-1004, c/src/backend.h:9-13).
//
// Each job is rows x cols weights (Q4_K, Q6_K or Q8_0) times nb activation vectors. K-quant jobs take the caller's Q8_K
// blocks (cl_xq) and give the CPU backend's numbers bit for bit (rowdot.cuh); Q8_0 jobs take the float vectors in the CPU's
// summation order. The CPU backend's CLUTOR_FLOAT_MATH switch is not honoured: K-quants always use the integer path.
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/clb200.h"
#include "common.cuh"
#include "rowdot.cuh"

namespace clb {

constexpr int MV_THREADS = 256;
constexpr int MV_ROWS = 16;

// out[b * rows + r] = row r of w times activation b, for rows [16*blockIdx.x, +16). K-quant activations come as the
// reference's cl_q8k blocks (xq_aos) or as plain arrays (sqs [nb][cols], sdd [nb][cols / 256], sbs [nb][cols / 16]);
// accum: out = out + scale * value (a residual update) instead of out = value.
__global__ void __launch_bounds__(MV_THREADS) mv_kernel(const uint8_t *w, uint32_t type, int rows, int cols, int nb,
                                                          const uint8_t *xq_aos, const float *xf, float *out, int *err,
                                                          const int8_t *sqs = nullptr, const float *sdd = nullptr,
                                                          const int16_t *sbs = nullptr, int accum = 0, float scale = 1.f) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * MV_ROWS, R = min(MV_ROWS, rows - r0);
  const uint32_t rb = type == T_Q8_0 ? cols / 32 * 34u : cols / 256 * (type == T_Q4_K ? 144u : 210u);
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
  float *xs = reinterpret_cast<float *>(sm + 16);                              // Q8_0: [cols] floats
  int8_t *qs = reinterpret_cast<int8_t *>(sm + 16);                            // K-quants: [cols] int8 ...
  float *dd = reinterpret_cast<float *>(sm + 16 + cols);                       // ... [cols / 256] scales
  int16_t *bs = reinterpret_cast<int16_t *>(sm + 16 + cols + 4 * (cols / 256));   // ... [cols / 16] group sums
  uint8_t *wbuf = sm + 16 + ((static_cast<size_t>(cols) * 4 + 127) & ~size_t(127));
  const uint8_t *src = w + static_cast<size_t>(r0) * rb;
  const uint32_t lo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src) & 15u);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    const uint32_t n16 = (lo + R * rb + 15u) & ~15u;
    mbar_arrive_expect_tx(bar, n16);
    bulk_copy_g2s(wbuf, src - lo, n16, bar);
  }
  __syncthreads();
  const bool q80 = type == T_Q8_0;
  const int nblk = q80 ? cols / 32 : cols / 256;
  const RowShape rs = row_shape(q80 ? nblk : 4 * nblk);
  const int sub = lane / rs.LG, lig = lane % rs.LG;
  if (!mbar_wait_bounded(bar, 0)) { set_error(err, ERR_WAIT_COPY); return; }
  const uint8_t *wrows = wbuf + lo;
  for (int b = 0; b < nb; ++b) {
    __syncthreads();
    if (q80) {
      for (int j = tid; j < cols; j += MV_THREADS) xs[j] = xf[static_cast<size_t>(b) * cols + j];
    } else if (sqs) {
      const int4 *q4 = reinterpret_cast<const int4 *>(sqs + static_cast<size_t>(b) * cols);
      for (int j = tid; j < cols / 16; j += MV_THREADS) reinterpret_cast<int4 *>(qs)[j] = q4[j];
      for (int j = tid; j < cols / 256; j += MV_THREADS) dd[j] = sdd[static_cast<size_t>(b) * (cols / 256) + j];
      for (int j = tid; j < cols / 16; j += MV_THREADS) bs[j] = sbs[static_cast<size_t>(b) * (cols / 16) + j];
    } else {   // unpack the caller's cl_q8k blocks {float d; int8 qs[256]; int16 bsums[16]} (292 bytes each)
      const uint8_t *blocks = xq_aos + static_cast<size_t>(b) * (cols / 256) * 292;
      for (int j = tid; j < cols; j += MV_THREADS) qs[j] = static_cast<int8_t>(blocks[(j / 256) * 292 + 4 + (j % 256)]);
      for (int j = tid; j < cols / 256; j += MV_THREADS) dd[j] = *reinterpret_cast<const float *>(blocks + j * 292);
      for (int j = tid; j < cols / 16; j += MV_THREADS)
        bs[j] = *reinterpret_cast<const int16_t *>(blocks + (j / 16) * 292 + 260 + 2 * (j % 16));
    }
    __syncthreads();
    KQAct act;
    if (!q80) load_kq_act(type, qs, dd, bs, nblk, rs, lig, act);
    for (int base = warp * rs.RPW; base < R; base += (MV_THREADS / 32) * rs.RPW) {
      const int r = base + sub;
      const bool active = sub < rs.RPW && r < R;
      const uint8_t *row = wrows + static_cast<size_t>(active ? r : 0) * rb;
      const float v = q80 ? q80_row(row, nblk, rs, lig, sub * rs.LG, xs, active) : kq_row(type, row, nblk, rs, lig, sub * rs.LG, act, active);
      if (active && lig == 0) {
        float *o = out + static_cast<size_t>(b) * rows + r0 + r;
        *o = accum ? __fadd_rn(*o, __fmul_rn(scale, v)) : v;
      }
    }
  }
}

// ---- host side ---------------------------------------------------------------------------------------------------------------
namespace {

struct Backend {
  std::mutex mu;
  int device = -1;
  cudaStream_t stream = nullptr;
  int *err = nullptr;
  std::unordered_map<const void *, std::pair<uint8_t *, size_t>> weights;   // host pointer -> device copy, bytes
  uint8_t *buf = nullptr;
  size_t buf_cap = 0;
};
Backend &backend() {
  static Backend b;
  return b;
}

[[noreturn]] void die(const char *what, cudaError_t e) {
  fprintf(stderr, "clutor-b200 backend: %s: %s\n", what, cudaGetErrorString(e));
  abort();
}
void check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) die(what, e);
}

uint64_t rbytes(uint32_t t, int cols) { return t == T_Q8_0 ? cols / 32 * 34ull : cols / 256 * (t == T_Q4_K ? 144ull : 210ull); }

int be_supports(uint32_t type) { return type == T_Q4_K || type == T_Q6_K || type == T_Q8_0; }

void be_matvec_batch(const clb200_mv *jobs, int n) {
  Backend &B = backend();
  std::lock_guard<std::mutex> lock(B.mu);
  if (B.device < 0) {
    const char *e = getenv("CLUTOR_B200_DEVICE");
    B.device = e ? atoi(e) : 0;
    check(cudaSetDevice(B.device), "selecting the device");
    check(cudaStreamCreateWithFlags(&B.stream, cudaStreamNonBlocking), "creating a stream");
    check(cudaMalloc(&B.err, 16), "allocating the error word");
    check(cudaMemset(B.err, 0, 16), "clearing the error word");
    check(cudaFuncSetAttribute(mv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024), "kernel attribute");
  }
  check(cudaSetDevice(B.device), "selecting the device");
  // per job: device weights, activations in, results out
  struct Plan { uint8_t *w; size_t act_off, out_off; int nb; };
  std::vector<Plan> plans(n);
  size_t need = 0;
  for (int j = 0; j < n; ++j) {
    const clb200_mv &m = jobs[j];
    const size_t wb = static_cast<size_t>(m.rows) * rbytes(m.type, m.cols);
    auto it = B.weights.find(m.w);
    if (it == B.weights.end() || it->second.second != wb) {
      if (it != B.weights.end()) cudaFree(it->second.first);
      uint8_t *d = nullptr;
      check(cudaMalloc(&d, wb + 64), "allocating weights");
      check(cudaMemcpy(d, m.w, wb, cudaMemcpyHostToDevice), "uploading weights");
      B.weights[m.w] = {d, wb};
    }
    plans[j].w = B.weights[m.w].first;
    plans[j].nb = m.nb > 1 ? (m.nb > 512 ? 512 : m.nb) : 1;
    plans[j].act_off = need;
    need += (m.type == T_Q8_0 ? static_cast<size_t>(m.cols) * 4 : static_cast<size_t>(m.cols / 256) * 292) * plans[j].nb;
    need = (need + 255) & ~size_t(255);
    plans[j].out_off = need;
    need += static_cast<size_t>(m.rows) * 4 * plans[j].nb;
    need = (need + 255) & ~size_t(255);
  }
  if (need > B.buf_cap) {
    check(cudaStreamSynchronize(B.stream), "waiting for the device");
    if (B.buf) cudaFree(B.buf);
    B.buf_cap = need * 2;
    check(cudaMalloc(&B.buf, B.buf_cap), "allocating activation buffers");
  }
  for (int j = 0; j < n; ++j) {
    const clb200_mv &m = jobs[j];
    const Plan &p = plans[j];
    uint8_t *act = B.buf + p.act_off;
    float *out = reinterpret_cast<float *>(B.buf + p.out_off);
    if (m.type == T_Q8_0) {
      const size_t pitch = (p.nb > 1 ? m.xf_stride : static_cast<size_t>(m.cols)) * 4;
      check(cudaMemcpy2DAsync(act, m.cols * 4, m.xf, pitch, m.cols * 4, p.nb, cudaMemcpyHostToDevice, B.stream), "copying activations");
    } else {
      const size_t blk = static_cast<size_t>(m.cols / 256) * 292;
      for (int b = 0; b < p.nb; ++b)
        check(cudaMemcpyAsync(act + b * blk, m.xq[b].b, blk, cudaMemcpyHostToDevice, B.stream), "copying activations");
    }
    const int grid = (m.rows + MV_ROWS - 1) / MV_ROWS;
    const size_t smem = 16 + ((static_cast<size_t>(m.cols) * 4 + 127) & ~size_t(127)) + ((MV_ROWS * rbytes(m.type, m.cols) + 32 + 15) & ~size_t(15)) + 16;
    mv_kernel<<<grid, MV_THREADS, smem, B.stream>>>(p.w, m.type, m.rows, m.cols, p.nb, m.type == T_Q8_0 ? nullptr : act,
                                                    m.type == T_Q8_0 ? reinterpret_cast<const float *>(act) : nullptr, out, B.err);
    check(cudaGetLastError(), "launching the product kernel");
    const size_t opitch = (p.nb > 1 ? m.out_stride : static_cast<size_t>(m.rows)) * 4;
    check(cudaMemcpy2DAsync(m.out, opitch, out, m.rows * 4, m.rows * 4, p.nb, cudaMemcpyDeviceToHost, B.stream), "copying results");
  }
  check(cudaStreamSynchronize(B.stream), "running the products");
  int code = 0;
  check(cudaMemcpy(&code, B.err, 4, cudaMemcpyDeviceToHost), "reading the error word");
  if (code) { fprintf(stderr, "clutor-b200 backend: device error %d\n", code); abort(); }
}

const clb200_backend_t kBackend = {"b200", be_supports, be_matvec_batch};

}  // namespace

size_t mv_smem_bytes(uint32_t type, int cols) {
  return 16 + ((static_cast<size_t>(cols) * 4 + 127) & ~size_t(127)) + ((MV_ROWS * rbytes(type, cols) + 32 + 15) & ~size_t(15)) + 16;
}

int launch_mv_dev(const uint8_t *w, uint32_t type, int rows, int cols, int nb, const int8_t *qs, const float *dd,
                  const int16_t *bs, float *out, int accum, float scale, int *err, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(mv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set[dev] = true;
  }
  const size_t smem = mv_smem_bytes(type, cols);
  if (smem > 200 * 1024) return static_cast<int>(cudaErrorInvalidValue);
  mv_kernel<<<(rows + MV_ROWS - 1) / MV_ROWS, MV_THREADS, smem, st>>>(w, type, rows, cols, nb, nullptr, nullptr, out, err, qs, dd, bs,
                                                                     accum, scale);
  return static_cast<int>(cudaGetLastError());
}
}  // namespace clb

extern "C" const clb200_backend_t *clb200_backend(void) { return &clb::kBackend; }
