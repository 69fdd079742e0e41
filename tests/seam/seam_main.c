/*
 * TEST DRIVER (not product code): the reference engine's own greedy decode loop (cl_fwd_open / cl_fwd_step,
 * c/src/forward.h:113-117) on a GGUF file, with its matrix products on the CPU backend or on clutor-b200's "b200" backend
 * registered through the reference's plugin seam (c/src/backend.h:9-19, c/src/quant.c:977-1004). Linked with the
 * reference's sources (tests/seam/Makefile) -- unmodified, or with forward.c carrying INTEGRATION.md's MoE hook.
 *
 *   seam_{ref,hook} <model.gguf> <steps> <cpu|b200> <out.bin>
 *
 * Writes steps x n_vocab float logits, then the steps greedy tokens (int32), to out.bin. Exits 0 on success.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "backend.h"
#include "clb200.h"
#include "forward.h"

int main(int argc, char **argv) {
  if (argc != 5) { fprintf(stderr, "usage: %s model.gguf steps cpu|b200 out.bin\n", argv[0]); return 2; }
  const int steps = atoi(argv[2]);
  if (!strcmp(argv[3], "b200")) {   /* the seam: register the backend, select it by name */
    if (!cl_backend_register((const cl_backend *)clb200_backend()) || !cl_backend_select("b200")) {
      fprintf(stderr, "registering the b200 backend failed\n");
      return 1;
    }
  } else if (!cl_backend_select("cpu")) {
    fprintf(stderr, "no cpu backend\n");
    return 1;
  }
  static cl_fwd f;
  char err[512] = {0};
  if (cl_fwd_open(&f, argv[1], steps + 8, NULL, err, sizeof err)) { fprintf(stderr, "open: %s\n", err); return 1; }
  const int V = f.n_vocab;
  float *logits = malloc((size_t)steps * V * sizeof(float));
  int32_t *toks = malloc((size_t)steps * sizeof(int32_t));
  if (!logits || !toks) return 1;
  int tok = 1;
  for (int s = 0; s < steps; s++) {
    float *lg = logits + (size_t)s * V;
    if (cl_fwd_step(&f, tok, lg, NULL, err, sizeof err)) { fprintf(stderr, "step %d: %s\n", s, err); return 1; }
    int best = 0;
    for (int i = 1; i < V; i++) if (lg[i] > lg[best]) best = i;
    toks[s] = tok = best;
  }
  FILE *o = fopen(argv[4], "wb");
  if (!o || fwrite(logits, sizeof(float), (size_t)steps * V, o) != (size_t)steps * V || fwrite(toks, sizeof(int32_t), steps, o) != (size_t)steps) {
    fprintf(stderr, "writing %s failed\n", argv[4]);
    return 1;
  }
  fclose(o);
  printf("%s: %d steps, backend %s, first tokens %d %d %d\n", argv[0], steps, cl_backend_active()->name, toks[0],
         steps > 1 ? toks[1] : -1, steps > 2 ? toks[2] : -1);
  cl_fwd_close(&f);
  free(logits);
  free(toks);
  return 0;
}
