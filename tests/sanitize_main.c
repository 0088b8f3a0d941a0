/* TEST INFRASTRUCTURE ONLY: drives the C host code (cwen_b200/host/*.c) over
 * the toy engine of tests/fake_engine.c under AddressSanitizer +
 * UndefinedBehaviorSanitizer ("host") or ThreadSanitizer ("threads"); built
 * and run by tests/test_sanitizers.py.  Exit status 0 when every step
 * behaved; a sanitizer report exits non-zero by itself. */
#define _GNU_SOURCE
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "cwen_host.h"
#include "synth.h"

int fake_config(int V, int P, int Q, int ctx);
int fake_config_mtp(int on);

static uint64_t rs = 0x9E3779B97F4A7C15ull;
static uint64_t rnd(void) {
  rs ^= rs << 13;
  rs ^= rs >> 7;
  rs ^= rs << 17;
  return rs;
}

#define CHECK(c)                                              \
  do {                                                        \
    if (!(c)) {                                               \
      fprintf(stderr, "check failed: %s (line %d)\n", #c, __LINE__); \
      return 1;                                               \
    }                                                         \
  } while (0)

static int read_file(const char *p, unsigned char **buf, long *n) {
  FILE *f = fopen(p, "rb");
  if (!f) return -1;
  fseek(f, 0, SEEK_END);
  *n = ftell(f);
  fseek(f, 0, SEEK_SET);
  *buf = malloc((size_t)*n + 1);
  size_t got = fread(*buf, 1, (size_t)*n, f);
  fclose(f);
  return got == (size_t)*n ? 0 : -1;
}
static int write_file(const char *p, const unsigned char *buf, long n) {
  FILE *f = fopen(p, "wb");
  if (!f) return -1;
  size_t put = fwrite(buf, 1, (size_t)n, f);
  return fclose(f) || put != (size_t)n ? -1 : 0;
}

static int gen_cb(void *user, const int32_t *t, int n_tok, int n_gen, int32_t *out) {
  return cwen_generate(t, n_tok, n_gen, out, (const cwen_spec_cfg *)user, NULL);
}

static int host(const char *dir) {
  char p[4096], q[4096];
  /* GGUF: write, probe, mutate */
  cwen_dims d, got;
  cwen_dims_small(&d);
  d.has_mtp = 1;
  snprintf(p, sizeof p, "%s/m.gguf", dir);
  CHECK(cwen_write_synth_gguf(p, &d, 7, 2) == 0);
  CHECK(cwen_gguf_dims(p, &got) == 0 && !memcmp(&got, &d, sizeof d));
  CHECK(cwen_load_gguf(p) == CWEN_ESTATE);
  unsigned char *base;
  long n;
  CHECK(read_file(p, &base, &n) == 0);
  unsigned char *b = malloc((size_t)n);
  snprintf(q, sizeof q, "%s/fz.gguf", dir);
  for (int it = 0; it < 300; it++) {
    memcpy(b, base, (size_t)n);
    long len = n;
    const long head = n < 8192 ? n : 8192;
    if (it % 3 == 0) {
      for (int j = 0; j < 4; j++) b[rnd() % (uint64_t)head] ^= (unsigned char)(1 + rnd() % 255);
    } else if (it % 3 == 1) {
      uint64_t v = rnd() >> (rnd() % 64);
      memcpy(b + 4 + rnd() % (uint64_t)(head - 12), &v, 8);
    } else {
      len = (long)(rnd() % (uint64_t)n);
    }
    CHECK(write_file(q, b, len) == 0);
    const int rc = cwen_gguf_dims(q, &got);
    CHECK(rc == 0 || rc == CWEN_EINVAL || rc == CWEN_ENOMEM);
  }
  free(b);
  free(base);
  /* the counted n-gram map and NGC2 */
  enum { HN = 3000 };
  int32_t *h = malloc(sizeof(int32_t) * HN);
  for (int i = 0; i < HN; i++) h[i] = (i % 37) * 1000 + (rnd() % 20 == 0 ? (int32_t)(rnd() % 900) : 0);
  cwen_ngram_map *m = cwen_ngram_map_new(4);
  CHECK(m != NULL);
  int32_t out[300];
  for (int hn = 8; hn < HN; hn += 13) {
    cwen_ngram_map_update(m, h, hn - 13 < 0 ? 0 : hn - 13, hn);
    CHECK(cwen_ngram_map_draft(m, h, hn, out, 15) >= 0);
    CHECK(cwen_ngram_draft(h, hn, out, 4, 300) >= 0);
  }
  snprintf(p, sizeof p, "%s/m.ngc", dir);
  CHECK(cwen_ngram_map_save(m, p, 248320) == 0);
  cwen_ngram_map_free(m);
  CHECK(read_file(p, &base, &n) == 0);
  b = malloc((size_t)n);
  snprintf(q, sizeof q, "%s/fz.ngc", dir);
  for (int it = 0; it < 100; it++) {
    memcpy(b, base, (size_t)n);
    long len = n;
    if (it % 2) b[rnd() % (uint64_t)n] ^= (unsigned char)(1 + rnd() % 255);
    else len = (long)(rnd() % (uint64_t)n);
    CHECK(write_file(q, b, len) == 0);
    m = cwen_ngram_map_new(4);
    CHECK(cwen_ngram_map_load(m, q, 248320) >= 0);
    CHECK(cwen_ngram_map_draft(m, h, HN, out, 15) >= 0);
    cwen_ngram_map_free(m);
  }
  free(b);
  free(base);
  /* the drivers over the toy engine, serial, n-gram and MTP speculation */
  int32_t prompt[200], res[400];
  for (int i = 0; i < 200; i++) prompt[i] = (int32_t)((i % 37) + (rnd() % 20 == 0 ? rnd() % 10 : 0)) % 50;
  cwen_spec_cfg cfg;
  for (int mode = 0; mode < 3; mode++) {
    CHECK(fake_config(50, 7, 3, mode == 2 ? 260 : 4096) == 0);
    fake_config_mtp(mode == 1);
    cwen_spec_defaults(&cfg);
    cfg.spec = 0;
    const int ns = cwen_generate(prompt, 200, 300, res, &cfg, NULL);
    CHECK(ns > 0);
    cfg.spec = 1;
    cfg.use_mtp = mode == 1;
    cfg.n_key = 4;
    cfg.min_draft = 1;
    cwen_spec_stats st;
    CHECK(cwen_generate(prompt, 200, 300, res, &cfg, &st) >= ns);
  }
  /* the frame server over pipes */
  fake_config(50, 7, 3, 512);
  fake_config_mtp(0);
  cwen_spec_defaults(&cfg);
  cfg.spec = 1;
  cfg.n_key = 4;
  int in[2], outp[2];
  CHECK(pipe(in) == 0 && pipe(outp) == 0);
  uint32_t frames[64];
  int k = 0;
  frames[k++] = 3; frames[k++] = 5; frames[k++] = 1; frames[k++] = 2; frames[k++] = 3;   /* valid */
  frames[k++] = 0; frames[k++] = 5;                                                      /* bad count */
  frames[k++] = 2; frames[k++] = 4; frames[k++] = 7; frames[k++] = 9999;                 /* bad id */
  frames[k++] = 600; frames[k++] = 2;                                                    /* > ctx, no payload */
  CHECK(write(in[1], frames, (size_t)k * 4) == (ssize_t)k * 4);
  close(in[1]);
  CHECK(cwen_serve(in[0], outp[1], 512, 50, gen_cb, &cfg) == 0);
  close(in[0]);
  close(outp[1]);
  uint32_t rep[64];
  const ssize_t got_b = read(outp[0], rep, sizeof rep);
  close(outp[0]);
  CHECK(got_b == (ssize_t)((1 + 5 + 1 + 1 + 1) * 4) && rep[0] == 5 && rep[6] == 0 && rep[7] == 0 && rep[8] == 0);
  free(h);
  return 0;
}

static int threads(void) {
  /* the seeded generator's worker threads write disjoint block ranges */
  const int K = 4096, M = 4096;
  void *w = malloc((size_t)(K / 32) * 18 * M);
  cw_synth_q4_0(1, "tsan.q4", K, M, w, 8);
  cw_synth_q8_0(1, "tsan.q8", K, M / 2, w, 8);
  free(w);
  return 0;
}

int main(int argc, char **argv) {
  if (argc != 3) return 2;
  if (!strcmp(argv[1], "host")) return host(argv[2]);
  if (!strcmp(argv[1], "threads")) return threads();
  return 2;
}
