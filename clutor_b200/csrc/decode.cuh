// Arguments and limits of the one-token MoE kernel (decode.cu) and the batched kernels (batched.cu).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace clb {

constexpr int DECODE_THREADS = 512;
constexpr int DECODE_MAX_NE = 256;   // experts per layer the one-token kernel ranks
constexpr int DECODE_MAX_K = 32;     // experts used per token
constexpr int ROUTE_SMEM_MAX_NE = 256;   // SMART-ROUTE inside the one-token kernel: experts per layer

struct DecodeArgs {
  const float *x_in;
  float *x_out;                  // may equal x_in
  const float *norm, *router;
  const uint8_t *gate, *up, *down;
  uint64_t gate_slab, up_slab, down_slab;
  uint32_t gate_type, up_type, down_type;
  int E, FF, NE, K, norm_topk;
  float resid_scale, eps;
  float *logits;                 // [NE] scratch ([2 NE] with router-ahead)
  float *hg;                     // [K * FF] scratch
  int *sel_out;                  // [K] or null
  float *wt_out;                 // [K] or null
  uint32_t *sync;                // [0] logits written, [1] CTAs whose hg rows are written, [2] CTAs finished; zero on entry
  int *err;                      // first device error
  int *err_out;                  // null, or host-mapped: the last CTA out copies the error word there (a host call reads it
                                 // after its one wait instead of copying it back)
  // 0: the whole block; 1: routing only (sel_out / wt_out; x unchanged); 2: the experts of a given routing (sel_in / wt_in,
  // renormalised already), each expert's weights at slab[k] (gate, up and down slabs back to back) or, where slab[k] is
  // null, in gate / up / down
  int mode;
  // test hook (0: off): the wait for the router logits targets a count that no CTA reaches, polled `stall_wait` times, so it
  // runs out and the launch reports ERR_WAIT_ROUTER without a hang or a fault
  uint32_t stall_wait;
  // test hook (mode 0): the copies of rank K - 1 first go out for the expert ranked K, so the slot correction runs
  int force_miss;
  int sel_in[DECODE_MAX_K];
  float wt_in[DECODE_MAX_K];
  const uint8_t *slab[DECODE_MAX_K];
  // shared-memory plan (host-computed): one slot per chosen expert holds this CTA's gate, up and down rows of it
  int rgu_max, rd_max;
  uint32_t grb, drb, gseg, dseg, slot_bytes;
  uint32_t off_bars, off_xn, off_norm, off_xq, off_router, off_rprod, off_misc, off_terms, off_hq, off_xr, off_slots, smem_bytes;
  // SMART-ROUTE in mode 1 (resident null: off): the residency of the layer's experts ([NE] bytes, device-visible), the
  // settings (c/src/route.h:14) and the counters of the routing (a RouteStats, device-visible), written by CTA 0
  const uint8_t *resident;
  int smart_J, smart_M;
  double smart_tau;
  void *smart_stats;
  // router-ahead in mode 1 (ahead_n 0: off; c/src/forward.c:937-946): the next layer's norm and router applied to this x
  // (logits to logits[NE, 2 NE)); CTA 0 writes the next layer's top ahead_n experts by logit, ties to the lower id, to
  // ahead_out (device-visible). Its rows and products use the expert slots, which routing-only launches leave free.
  const float *ahead_norm, *ahead_router;
  int ahead_n;
  int *ahead_out;
  // phase trace (null: off): thread 0 of CTA c writes its SM's cycle counter at phase boundary i to trace[32 * c + i] and the global
  // nanosecond timer at entry and exit to trace[32 * c + 30] and [31]
  unsigned long long *trace;
};

// The one-token kernel for experts of these types (gate/up share one type), or null when it has none.
using DecodeFn = void (*)(DecodeArgs);
// n floats (n a multiple of 4, at most 4096) from host-mapped src to device dst on st, by one small CTA that lets the next
// kernel launch at once (programmatic dependent launch): a host call's x reaches the one-token kernel without a
// copy-engine transfer.
cudaError_t launch_stage_in(const float *src, float *dst, int n, cudaStream_t st);
DecodeFn decode_kernel_for(uint32_t gate_type, uint32_t down_type);
// Lets every instantiation use `bytes` of dynamic shared memory (on the current device).
cudaError_t decode_allow_smem(int bytes);

// ---- the expert-group one-token kernel (group.cu) -----------------------------------------------------------------------
constexpr int GROUP_THREADS = 512;
constexpr int GROUP_MAX_RG = 31;   // gate/up row groups per CTA (one mbarrier and one copy pair each)
constexpr int GROUP_MAX_NE = 256;

struct GroupArgs {
  const float *x_in;
  float *x_out;                  // may equal x_in
  const float *norm, *router;
  const uint8_t *gate, *up, *down;
  uint64_t gate_slab, up_slab, down_slab;
  int E, FF, NE, K, norm_topk;
  float resid_scale, eps;
  // the kernel's own exchange buffer (zero when first used, written by nothing else): sync [0] the launch generation; lw [NE]
  // logit words; hw [K * FF] hg words, then [K * E] words of each group's weighted down rows
  uint32_t *sync;
  unsigned long long *lw, *hw;
  int *err;                      // first device error
  int *err_out;                  // null, or host-mapped: the last CTA out copies the error word there
  int *sel_out;                  // [K] or null
  float *wt_out;                 // [K] or null
  int force_miss;                // test hook: the copies of rank K - 1 first go out for the expert ranked K, so the correction runs
  // plan (host-computed, plan_group_shape)
  int ne;                        // CTAs per expert group; the grid is K * ne workers plus CTAs that only score experts
  int GL;                        // lanes per gate/up row (a power of two >= E / 256)
  int nrg_max, ngu_max, nd_max, nre;
  uint32_t grb, drb, rg_bytes, rstride;
  uint32_t off_bars, off_x, off_norm, off_xn, off_xq, off_router, off_prod, off_lg, off_ev, off_p, off_misc, off_hg, off_hq,
      off_terms, off_own, off_gath, off_gu, off_dn, smem_bytes;
  unsigned long long *trace;     // as DecodeArgs::trace
};
using GroupFn = void (*)(GroupArgs);
// Bytes of the exchange buffer a layer of this shape needs.
size_t group_buffer_bytes(int sms, int E, int FF, int NE, int K);
// The plan for a layer on a device with `sms` SMs and `max_smem` bytes of opt-in shared memory; 0 when the kernel takes it.
int plan_group_shape(int sms, int max_smem, int E, int FF, int NE, int K, uint32_t gate_type, uint32_t up_type,
                     uint32_t down_type, GroupArgs &a);
GroupFn group_kernel_for(uint32_t gate_type, uint32_t down_type);
cudaError_t group_allow_smem(int bytes);
// Points the args at an exchange buffer of group_buffer_bytes() bytes (laid out by a.NE, a.K, a.FF and a.E: set them first).
void group_set_buffer(GroupArgs &a, uint8_t *buf, int sms);

// ---- batched path ------------------------------------------------------------------------------------------------------
struct BatchArgs {
  const float *x_in;
  float *x_out;
  const float *norm, *router;
  const uint8_t *gate, *up, *down;
  uint64_t gate_slab, up_slab, down_slab;
  uint32_t gate_type, up_type, down_type;
  int T, E, FF, NE, K, norm_topk;
  float resid_scale, eps;
  uint32_t grb, drb;
  // scratch
  float *xn;            // [T * E]
  int8_t *xq_qs;        // [T * E]
  float *xq_d;          // [T * E / 256]
  int16_t *xq_bs;       // [T * E / 16]
  float *logits;        // [T * NE]
  int *sel;             // [T * K]
  float *wt;            // [T * K]
  int *counts;          // [NE]
  int *offsets;         // [NE + 1]
  int *first;           // [NE] first appearance (slot index t*K+k) of each expert
  int *todo;            // [NE + 1] the experts with tokens in order of first appearance (the reference's todo[]), their count
                        // at [NE]
  int *pos_token;       // [T * K] dispatch position -> token
  float *pos_wt;        // [T * K] dispatch position -> routing weight
  int *slot_pos;        // [T * K] (t, k) -> dispatch position
  float *hg;            // [T * K * FF] by dispatch position
  int8_t *hq_qs;        // [T * K * FF]
  float *hq_d;          // [T * K * FF / 256]
  int16_t *hq_bs;       // [T * K * FF / 16]
  float *hd;            // [T * K * E] by dispatch position
  __half *xh, *xl;      // [T * E] xn as fp16 hi and lo planes (tensor-core path; null otherwise)
  __half *hgh, *hgl;    // [T * K * FF] hg as fp16 hi and lo planes, by dispatch position (tensor-core path)
  __half *xdh, *xdl;    // [T * K * E] the xn planes gathered into dispatch order (tensor-core path)
  int *sel_out;         // [T * K] or null
  float *wt_out;        // [T * K] or null
  int *err;
  // expert-parallel expert side: sel entries may be -1 (an expert another GPU holds); the dispatch leaves them out and
  // the combine writes the weighted sum of the present experts alone (x_out = moe, no residual, x_in unused)
  int ep;
  // tensor-core expert products (grouped_tc.cu) for gate/up and for down
  int tc_gu, tc_dn;
  // [T * K] the power of two each dispatch row of the current K-quant activation planes was divided by (so that the fp16
  // planes hold any Q8_K row without overflow); the tensor-core epilogue multiplies it back. Null: no scaling (Q8_0).
  float *rs;
};

// Launches the batched path on `stream`; returns a CUDA error code.
int launch_batched(const BatchArgs &a, void *stream);
// Its two halves: rmsnorm + Q8_K + router + top-k (sel / wt), and everything from the dispatch on (given sel / wt / xq).
int launch_route(const BatchArgs &a, void *stream);
int launch_experts(const BatchArgs &a, void *stream);
// The dispatch alone (sel / wt -> counts, offsets, first, todo, pos_token, pos_wt, slot_pos).
int launch_dispatch(const BatchArgs &a, void *stream);
// The Q8_0 / Q4_K expert products on tcgen05 (grouped_tc.cu): gate/up (writes hg, and hgh/hgl for Q8_0 down) or down
// (writes hd).
int launch_tc(const BatchArgs &a, void *stream, bool gateup);
// A dense Q4_K matrix times nb tokens' plain Q8_K rows on the tensor cores (grouped_tc.cu): out [nb][rows]; co holds the
// device ints {nb, 0, nb}; ph / pl [nb][cols] halves and rs [nb] are scratch. Returns a CUDA error code.
int launch_tc_dense(const uint8_t *w, uint32_t rb, int rows, int cols, int nb, const int8_t *qs, const float *dd, int *co,
                    __half *ph, __half *pl, float *rs, float *out, int *err, cudaStream_t st);
// Whether the tensor-core path takes experts of this type at w (Q8_0 or Q4_K, 16-byte aligned, E and FF multiples of 256).
bool tc_type_supported(uint32_t type, const void *w, int E, int FF);

}  // namespace clb
