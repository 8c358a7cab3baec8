/*
 * Driver for the reference's own CPU FP32 build (gpt2.c compiled from the
 * reference tree with -Dmain=gpt2_reference_main). Runs the reference's main
 * unchanged, then optionally writes one row of its global logits buffer
 * (gpt2.c: act_t logits[ctx_len][vocab_size], fp32 in this build) to a file.
 * Test infrastructure only.
 *
 * usage: gpt2_ref_<size> [--dump-logits FILE ROW] <gpt2.c arguments...>
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define REF_VOCAB 50257
#define REF_CTX 1024

int gpt2_reference_main(int argc, char **argv);
#ifndef REF_NO_LOGITS
extern float logits[REF_CTX][REF_VOCAB];
#endif

int main(int argc, char **argv) {
  const char *dump = NULL;
  int row = -1;
  int first = 1;
  if (argc >= 4 && strcmp(argv[1], "--dump-logits") == 0) {
    dump = argv[2];
    row = atoi(argv[3]);
    first = 4;
  }
  char **args = (char **)malloc(sizeof(char *) * (size_t)(argc - first + 2));
  int n = 0;
  args[n++] = argv[0];
  for (int i = first; i < argc; ++i) args[n++] = argv[i];
  args[n] = NULL;
  int rc = gpt2_reference_main(n, args);
  free(args);
#ifdef REF_NO_LOGITS
  if (dump) return 5; /* GPU builds: the logits live on the device */
#endif
  if (rc == 0 && dump) {
    if (row < 0 || row >= REF_CTX) return 3;
    FILE *fp = fopen(dump, "wb");
    if (!fp) return 4;
#ifndef REF_NO_LOGITS
    fwrite(logits[row], sizeof(float), REF_VOCAB, fp);
#endif
    fclose(fp);
  }
  return rc;
}
