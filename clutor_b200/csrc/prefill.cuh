// The batched prompt path of the whole model (prefill.cu): the reference's run_std (c/src/forward.c:1078-1225) for the
// mixture-of-experts architectures, as a sequence of kernels per layer over a batch of nb tokens. The dense products run
// through the product kernel of backend.cu (launch_mv_dev) and the MoE block through the batched path (batched.cu,
// grouped_tc.cu); the kernels here are the per-token steps between them.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "fwd.cuh"

namespace clb {

constexpr int PF_MAX_BATCH = 512;   // CL_PS_B (c/src/forward.h:121)
constexpr int PF_MAX_CTX = 32768;   // positions a batched attention item keeps in shared memory

// X [nb][E] = the embedding rows of tok [nb] (device), times embed_scale.
cudaError_t pf_embed(const FwdMat &emb, const int *tok, int nb, int E, float embed_scale, float *X, cudaStream_t st);
// rmsnorm of rows [row0, row0 + nb) of X [.][E] with weights w, then Q8_K in plain layout: qs [nb][E], dd [nb][E / 256],
// bs [nb][E / 16] (c/src/forward.c:412-417, c/src/quant.c:195-206).
cudaError_t pf_norm_q8k(const float *X, int row0, int nb, int E, const float *w, float eps, int8_t *qs, float *dd, int16_t *bs,
                        cudaStream_t st);
// Q8_K in plain layout of nb rows of `cols` floats.
cudaError_t pf_q8k(const float *src, int nb, int cols, int8_t *qs, float *dd, int16_t *bs, cudaStream_t st);
// Per token b (position pos0 + b): QK-norm and the rotary embedding of its query heads (Q [nb][n_q] -> Qr) and key heads,
// and its key and value stored in layer l's half-precision cache (c/src/forward.c:1100-1118).
struct PfQkArgs {
  const float *Q, *K, *V;    // [nb][n_q], [nb][n_kvw], [nb][n_kvw]
  float *Qr;                 // [nb][n_q]
  const float *qn, *kn;      // QK-norm weights (null without)
  __half *kc, *vc;           // layer l's cache: [ctx][n_kvw]
  const float *rope_cs;      // [ctx][hd]
  int nb, pos0, n_head, n_kv, hd, qk_mode, rope_pairs;
  float eps;
};
cudaError_t pf_qk(const PfQkArgs &a, cudaStream_t st);
// Attention of every (token, query head), one task each, as the reference's attn_task (c/src/forward.c:584-620): scores
// with dotf_h against every cached position up to the token's own, softmax with a float sum in position order, the values
// added in position order with weight score / sum.
struct PfAttnArgs {
  const float *Qr;           // [nb][n_q]
  const __half *kc, *vc;     // layer l's cache
  float *att;                // [nb][n_q]
  int nb, pos0, n_head, n_kv, hd, n_kvw;
  float attn_scale;
};
cudaError_t pf_attn(const PfAttnArgs &a, cudaStream_t st);

// A dense product of a batch, out [nb][rows] (= or += scale *) m [rows][cols] times plain Q8_K activations: a CTA per 32
// rows and 32 tokens for batches of 8 or more tokens, else the product kernel of backend.cu. Returns a CUDA error code.
int pf_mv(const FwdMat &m, int rows, int cols, int nb, const int8_t *qs, const float *dd, const int16_t *bs, float *out, int accum,
          float scale, int *err, cudaStream_t st);
// Scratch of the tensor-core dense products: the count/offsets triple, fp16 hi/lo activation planes [nb][cols], a power of
// two per token, and a product buffer [nb][rows] for products added into a residual.
struct PfTc {
  int *co;
  __half *ph, *pl;
  float *rs, *tmp;
};
// The same product with a Q4_K matrix on the tensor cores (fp16 hi/lo operands, ~1e-6 from the integer product) for
// batches of 256 or more tokens; other types and smaller batches through pf_mv. Returns a CUDA error code.
int pf_mv_tc(const FwdMat &m, int rows, int cols, int nb, const int8_t *qs, const float *dd, const int16_t *bs, float *out, int accum,
             float scale, const PfTc &tc, int *err, cudaStream_t st);
// The dense product kernel of backend.cu: out [nb][rows] (= or += scale *) w [rows][cols] times plain Q8_K activations.
int launch_mv_dev(const uint8_t *w, uint32_t type, int rows, int cols, int nb, const int8_t *qs, const float *dd,
                  const int16_t *bs, float *out, int accum, float scale, int *err, cudaStream_t st);

}  // namespace clb
