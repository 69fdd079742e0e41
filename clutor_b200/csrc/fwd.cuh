// The whole-model one-token step (fwd.cu): the reference's cl_fwd_step (c/src/forward.c:878-1040) for the mixture-of-experts
// transformer architectures (olmoe, qwen3moe, granitemoe) as ONE persistent kernel per token.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace clb {

constexpr int FWD_THREADS = 512;
constexpr int FWD_MAX_K = 16;       // experts used per token (one warp issues each expert's copies)
constexpr int FWD_MAX_NE = 128;     // experts per layer the kernel ranks (four threads per expert)
constexpr int FWD_ATT_CHUNK = 256;  // positions per attention chunk (the reference's ATT_CHUNK)
constexpr int FWD_ATT_BLOCK = 128;  // positions of keys or values staged in shared memory at once
constexpr int FWD_MAX_GROUP = 16;   // query heads per key/value head
constexpr int HEAD_ROWS = 24;       // output-matrix rows per shared-memory stage
constexpr int HEAD_STAGES = 4;      // stages in flight (they span the slots and the dslots); two are computed at a time

// A quantized weight matrix on the device, GGUF blocks as in the file: rows x cols, row r at p + r * rb.
struct FwdMat {
  const uint8_t *p;
  uint32_t type;
  uint32_t rb;   // bytes per row
};

// One layer's tensors on the device (the reference's cl_fwd_layer, c/src/forward.h:18-29).
struct FwdLayer {
  const float *attn_norm, *ffn_norm, *qn, *kn;   // fp32; qn / kn null without QK-norm
  const float *router;                           // fp32 [NE][E]
  FwdMat wq, wk, wv, wo;
  const uint8_t *gate, *up, *down;               // fused expert tensors
  uint32_t gate_type, down_type;                 // gate and up share a type
  uint64_t gate_slab, up_slab, down_slab;
};

// Host-written, device-updated state of the sequence: the next token to feed and its position. The step reads both and
// writes back the greedy choice (the arg-max of the logits, lowest id on ties, as c/src/main.c:349-350) and pos + 1.
struct FwdState {
  int token;
  int pos;
  int next;        // the token chosen by the last step
  int err;         // first device error (codes of common.cuh)
  unsigned long long best;   // arg-max key of the step in flight
  uint32_t sync[4];          // [0] grid barrier counter, [1] router logits, [2] exits
};

struct FwdArgs {
  // shape
  int E, n_head, n_kv, hd, n_q, n_kvw, FF, NE, K, vocab, n_layer, ctx;
  int qk_mode;      // 0 none, 1 whole vector (olmoe), 2 per head (qwen3moe)
  int norm_topk, rope_pairs, feed;
  float eps, rope_base, attn_scale, resid_scale, embed_scale, logit_scale;
  // weights
  FwdMat tok_embd, output;
  const float *out_norm;
  const FwdLayer *layers;
  // key/value cache [n_layer][ctx][n_kvw], half precision
  __half *kc, *vc;
  // scratch
  float *x;          // [E] the residual stream
  float *qkv;        // [n_q + 2 n_kvw]
  float *att;        // [n_q]
  float *rlogits;    // [NE] router logits
  float *hg;         // [K * FF]
  float *logits;     // [vocab]
  int *route_sel;    // [n_layer][K] the chosen experts of the last step, rank order
  float *route_wt;   // [n_layer][K] their weights
  int *gen_out;      // [ctx] the token chosen at each position
  FwdState *st;
  // per-CTA shared-memory plan (host-computed)
  uint32_t grb, drb, gseg, slot_bytes, dslot_bytes;
  uint32_t off_bars, off_xn, off_xq, off_misc, off_router, off_rprod, off_terms, off_hq, off_xr, off_slots, off_dslots, smem_bytes;
  const float *rope_cs;        // [ctx][hd]: per position hd / 2 cosines then hd / 2 sines of the rotary angles, as the
                               // reference computes them (c/src/forward.c:428-435)
  int rgu_max, rd_max, nre_max;
  unsigned long long *trace;   // per-CTA phase trace (32 entries per CTA) or null
  int force_miss;              // test hook: the copies of rank K - 1 first go out for the expert ranked K (0: off)
};

// Launches one step on `stream` with `ctas` CTAs (one per SM, all co-resident: a cooperative launch).
cudaError_t fwd_launch(const FwdArgs &a, int ctas, cudaStream_t stream);
cudaError_t fwd_allow_smem(int bytes);

}  // namespace clb
