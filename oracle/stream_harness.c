/* Test infrastructure: exports the reference stress harness's synthetic router (c/src/stream.c:114-140, static there) so
 * the tests can pin this repository's restatement of it (clutor_b200.synth.ExpertStream) value for value. */
#include "stream.c"

void *ref_stream_new(int L, int E, double locality, unsigned long long seed, double rho) {
  router *r = malloc(sizeof *r);
  if (r) router_init(r, L, E, locality, (uint64_t)seed, rho);
  return r;
}
void ref_stream_logits(void *r, long t, int l, int predicted, int mode, float *out) { router_logits((router *)r, t, l, predicted, mode, out); }
void ref_stream_free(void *r) {
  router *p = r;
  if (!p) return;
  free(p->base);
  free(p->bonus);
  free(p);
}
