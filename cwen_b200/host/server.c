/* Binary-frame server of the C host (CWEN_SERVER=1): the request/reply loop
 * of server_loop (run.c:5063-5078) with the framing checks of
 * server_read_frame (run.c:4216-4235).
 *
 * Request: u32 n_prompt, u32 n_gen, n_prompt x int32 token ids (little
 * endian).  Reply: u32 n_out, n_out x int32 generated ids.  A frame with
 * n_prompt or n_gen outside [1, ctx] gets the reply 0 and its declared
 * payload is consumed, so the next header stays aligned; a frame with a
 * token id outside [0, n_vocab) gets the reply 0.  End of input -- between
 * frames or inside one -- ends the loop cleanly.  Generation itself is the
 * caller's function, which the CLI points at cwen_generate (state reset and
 * prefill per request, serial or speculative per the knobs).
 */
#define _GNU_SOURCE
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "cwen_host.h"
#include "host_err.h"

/* 0xffffffff also when the read fails (the reference's end-of-input value) */
static uint32_t rd_u32(FILE *f) {
  uint32_t v = 0;
  return fread(&v, 4, 1, f) == 1 ? v : 0xffffffffu;
}

static void drain(FILE *f, uint64_t n) {
  uint32_t buf[1024];
  while (n) {
    const size_t take = n > 1024 ? 1024 : (size_t)n;
    if (fread(buf, 4, take, f) != take) return;
    n -= take;
  }
}

static int reply(FILE *f, const int32_t *t, uint32_t n) {
  if (fwrite(&n, 4, 1, f) != 1 || (n && fwrite(t, 4, n, f) != n) || fflush(f))
    return host_fail(CWEN_EINVAL, "cwen server: reply write failed");
  return CWEN_OK;
}

int cwen_serve(int in_fd, int out_fd, int ctx, int n_vocab, cwen_generate_fn gen, void *user) {
  if (in_fd < 0 || out_fd < 0 || ctx < 1 || n_vocab < 1 || !gen)
    return host_fail(CWEN_EINVAL, "cwen_serve: bad arguments");
  const int ifd = dup(in_fd), ofd = dup(out_fd);
  FILE *in = ifd >= 0 ? fdopen(ifd, "rb") : NULL;
  FILE *out = ofd >= 0 ? fdopen(ofd, "wb") : NULL;
  int32_t *toks = (int32_t *)malloc(sizeof(int32_t) * (size_t)ctx);
  int32_t *res = (int32_t *)malloc(sizeof(int32_t) * (size_t)ctx);
  int rc = CWEN_OK;
  if (!in || !out || !toks || !res) {
    rc = host_fail(CWEN_ENOMEM, "cwen_serve: %s", strerror(errno ? errno : ENOMEM));
    goto done;
  }
  for (;;) {
    const uint32_t np = rd_u32(in), ng = rd_u32(in);
    if (np == 0xffffffffu || ng == 0xffffffffu) break;  /* end of input */
    if (!np || np > (uint32_t)ctx || !ng || ng > (uint32_t)ctx) {
      fprintf(stderr, "cwen server: bad frame %u %u\n", np, ng);
      drain(in, np);
      if ((rc = reply(out, NULL, 0))) break;
      continue;
    }
    if (fread(toks, 4, np, in) != np) break;  /* end of input inside the payload */
    uint32_t bad = np;
    for (uint32_t i = 0; i < np && bad == np; i++)
      if (toks[i] < 0 || toks[i] >= n_vocab) bad = i;
    if (bad < np) {
      fprintf(stderr, "cwen server: token %d out of range [0,%d)\n", toks[bad], n_vocab);
      if ((rc = reply(out, NULL, 0))) break;
      continue;
    }
    const int n = gen(user, toks, (int)np, (int)ng, res);
    if (n < 0) {
      rc = n;
      break;
    }
    if ((rc = reply(out, res, (uint32_t)n))) break;
  }
done:
  free(toks);
  free(res);
  if (in) fclose(in);
  else if (ifd >= 0) close(ifd);
  if (out) fclose(out);
  else if (ofd >= 0) close(ofd);
  return rc;
}
