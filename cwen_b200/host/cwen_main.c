/* cwen CLI on the B200 engine: the reference's command line (run.c:5081-5251)
 *
 *   cwen [MODEL] [IDS_FILE] [N_PREDICT] [-d N]
 *
 * MODEL is a GGUF file, or "synth:SEED" / "synth:SEED:small" for the seeded
 * random-init model (no file).  IDS_FILE holds little-endian int32 ids.
 * Generated ids go to stdout, logs to stderr.  Knobs: CWEN_SPEC, CWEN_MTP,
 * CWEN_CTX (64..32768), CWEN_SPEC_NGRAM_N/MAX_DRAFT/MIN_DRAFT/COOLDOWN/DEBUG,
 * CWEN_NGRAM_CACHE, CWEN_SERVER (binary-frame server on stdin/stdout,
 * host/server.c), CWEN_DEVICE (GPU index), CWEN_REPACK (CWENR sidecar).
 */
#define _GNU_SOURCE
#include <errno.h>
#include <limits.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cwen_host.h"

static void usage(FILE *o) {
  fprintf(o,
          "usage: cwen [MODEL] [IDS_FILE] [N_PREDICT] [OPTIONS]\n"
          "Argmax-generate token ids from raw little-endian int32 prompt ids on a B200.\n"
          "  MODEL      GGUF path, or synth:SEED[:small] for the seeded random model\n"
          "  IDS_FILE   int32 token ids (omitted: the single token 248044)\n"
          "  N_PREDICT  tokens to generate, >= 0 (default 16)\n"
          "  -d, --draft-tokens N   speculate up to N drafts per verify block (1..15);\n"
          "                         implies CWEN_SPEC=1\n"
          "Environment:\n"
          "  CWEN_CTX=N             context window, 64..32768 (default 4096)\n"
          "  CWEN_DEVICE=N          GPU index (default 0)\n"
          "  CWEN_REPACK=FILE       CWENR sidecar (auto: MODEL with .cwenr)\n"
          "  CWEN_SERVER=1          binary-frame server on stdin/stdout\n"
          "  CWEN_SPEC=1            block speculation (greedy-lossless); drafter: the\n"
          "                         model's MTP nextn head when present, else the n-gram map\n"
          "  CWEN_MTP=0             do not draft with the MTP head\n"
          "  CWEN_NGRAM_CACHE=FILE  persist the n-gram map across runs (NGC2)\n"
          "    CWEN_SPEC_NGRAM_N=N      lookup key length (default 16)\n"
          "    CWEN_SPEC_MAX_DRAFT=N    max drafts per block, 1..15 (default 8)\n"
          "    CWEN_SPEC_MIN_DRAFT=N    skip blocks shorter than N drafts (default 2)\n"
          "    CWEN_SPEC_COOLDOWN=N     plain steps after repeated full rejects (8)\n"
          "    CWEN_SPEC_DEBUG=1        per-cycle speculation trace on stderr\n");
}

/* cwen_serve's generator: one request through the C driver. */
static int serve_generate(void *user, const int32_t *tokens, int n_tok, int n_gen, int32_t *out) {
  cwen_spec_stats st;
  return cwen_generate(tokens, n_tok, n_gen, out, (const cwen_spec_cfg *)user, &st);
}

static int arg_int(const char *a, long lo, long hi, const char *what) {
  char *end;
  long v = strtol(a, &end, 10);
  if (end == a || *end || v < lo || v > hi) {
    fprintf(stderr, "cwen: %s must be an integer in [%ld,%ld], got '%s'\n", what, lo, hi, a);
    exit(2);
  }
  return (int)v;
}

int main(int argc, char **argv) {
  const char *model = "model/Qwen3.8-27B-Q4_0.gguf", *ids = NULL;
  int n_predict = 16, draft = -1, npos = 0;
  const char *pos[3];
  for (int i = 1; i < argc; i++) {
    const char *a = argv[i];
    if (!strcmp(a, "-h") || !strcmp(a, "--help")) { usage(stdout); return 0; }
    if (a[0] == '-' && a[1]) {
      if (strcmp(a, "-d") && strcmp(a, "--draft-tokens") && strcmp(a, "--spec-draft-n-max")) {
        fprintf(stderr, "cwen: unknown option '%s'\n\n", a);
        usage(stderr);
        return 2;
      }
      if (i + 1 >= argc) { fprintf(stderr, "cwen: %s requires a value\n", a); return 2; }
      draft = arg_int(argv[++i], 1, 15, a);
      continue;
    }
    if (npos >= 3) { fprintf(stderr, "cwen: too many arguments\n"); usage(stderr); return 2; }
    pos[npos++] = a;
  }
  if (npos >= 1) model = pos[0];
  if (npos >= 2) ids = pos[1];
  if (npos >= 3) n_predict = arg_int(pos[2], 0, INT_MAX, "N_PREDICT");

  cwen_spec_cfg cfg;
  cwen_spec_defaults(&cfg);
  if (cwen_spec_from_env(&cfg)) return 1;
  int server = 0;  /* CWEN_SERVER: checked before the model load, like the reference */
  {
    const char *sv = getenv("CWEN_SERVER");
    if (sv && sv[0]) {
      if (strcmp(sv, "0") && strcmp(sv, "1")) { fprintf(stderr, "cwen: CWEN_SERVER must be 0 or 1\n"); return 1; }
      server = sv[0] == '1';
    }
  }
  if (draft > 0) {
    cfg.max_draft = draft;
    cfg.spec = 1;
    if (cfg.min_draft > cfg.max_draft) cfg.min_draft = cfg.max_draft;
  }
  int ctx = 4096, dev = 0;
  const char *e = getenv("CWEN_CTX");
  if (e && e[0]) ctx = arg_int(e, 64, 32768, "CWEN_CTX");
  e = getenv("CWEN_DEVICE");
  if (e && e[0]) dev = arg_int(e, 0, 255, "CWEN_DEVICE");
  fprintf(stderr, "ctx: %d\n", ctx);

  if (cwen_cuda_init(dev, ctx, 16)) {
    fprintf(stderr, "cwen: %s\n", cwen_cuda_last_error());
    return 1;
  }
  int rc;
  if (!strncmp(model, "synth:", 6)) {
    cwen_dims d;
    const char *s = model + 6;
    char *end;
    unsigned long long seed = strtoull(s, &end, 10);
    if (end == s) { fprintf(stderr, "cwen: bad synth seed in '%s'\n", model); return 2; }
    if (!strcmp(end, ":small")) cwen_dims_small(&d);
    else cwen_dims_reference(&d);
    rc = cwen_load_synth(seed, &d, 0);
  } else {
    rc = cwen_load_gguf(model);
  }
  if (rc) {
    fprintf(stderr, "cwen: load failed: %s\n", cwen_cuda_last_error());
    return 1;
  }
  if (server) {
    cwen_dims md;
    if (cwen_cuda_model_dims(&md)) { fprintf(stderr, "cwen: %s\n", cwen_cuda_last_error()); return 1; }
    fprintf(stderr, "cwen server: model loaded, waiting on stdin\n");
    rc = cwen_serve(0, 1, ctx, md.n_vocab, serve_generate, &cfg);
    if (rc) fprintf(stderr, "cwen: %s\n", cwen_cuda_last_error());
    cwen_cuda_shutdown();
    return rc ? 1 : 0;
  }
  int32_t *toks = (int32_t *)malloc(sizeof(int32_t) * (size_t)ctx);
  if (!toks) { fprintf(stderr, "cwen: out of host memory\n"); return 1; }
  int n_tok = 0;
  if (ids) {
    FILE *f = fopen(ids, "rb");
    if (!f) { perror(ids); return 1; }
    while (n_tok < ctx && fread(&toks[n_tok], 4, 1, f) == 1) n_tok++;
    fclose(f);
  } else {
    toks[0] = 248044;
    n_tok = 1;
  }
  if (n_tok < 1) { fprintf(stderr, "cwen: %s: no tokens in prompt\n", ids); return 1; }
  int32_t *out = (int32_t *)malloc(sizeof(int32_t) * (size_t)(n_predict ? n_predict : 1));
  if (!out) { fprintf(stderr, "cwen: out of host memory\n"); return 1; }
  fprintf(stderr, "prefill %d tokens...\n", n_tok);
  cwen_spec_stats st;
  int n = cwen_generate(toks, n_tok, n_predict, out, &cfg, &st);
  if (n < 0) {
    fprintf(stderr, "cwen: %s\n", cwen_cuda_last_error());
    return 1;
  }
  for (int i = 0; i < n; i++) printf(i ? " %d" : "%d", out[i]);
  if (n > 0) putchar('\n');
  cwen_cuda_shutdown();
  if (fflush(stdout) || ferror(stdout)) { fprintf(stderr, "cwen: stdout write failed\n"); return 1; }
  return 0;
}
