/* Decode drivers of the C host: prefill, serial greedy decode and greedy
 * block speculation, plus the n-gram prompt-lookup drafter.
 *
 * Semantics follow the reference's drivers (generate_tokens run.c:5027-5045,
 * generate_tokens_spec run.c:4882-5018, prefill_forward run.c:4823-4857):
 * the same cycle invariant, drafter choice, min_draft gate, AIMD draft cap,
 * rejection-streak cooldown and stats line.  What changes is the engine
 * underneath: a short walk commits the kept rows of the verify block on the
 * device (cwen_cuda_commit) instead of restoring a snapshot and re-scoring
 * them, and prefill chunks use the engine's full block width (its kernels
 * are batch-invariant, so the chunking cannot change a single bit).
 */
#define _GNU_SOURCE
#include <errno.h>
#include <limits.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cwen_host.h"
#include "host_err.h"

/* ---- knobs ---- */
void cwen_spec_defaults(cwen_spec_cfg *c) {
  if (!c) return;
  c->spec = 0;
  c->use_mtp = 1;
  c->max_draft = 8;
  c->min_draft = 2;
  c->n_key = 16;
  c->cooldown = 8;
  c->debug = 0;
}

/* A bad knob: reported on stderr, like the reference, and recorded for
   cwen_cuda_last_error(). */
static int env_fail(const char *fmt, ...) {
  char buf[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  fprintf(stderr, "cwen: %s\n", buf);
  cwen_host_set_error(buf);
  return CWEN_EINVAL;
}

static int env_int_strict(const char *name, int *out, int *rc) {
  const char *e = getenv(name);
  if (!e || !e[0]) return 0;
  char *end;
  long v = strtol(e, &end, 10);
  if (end == e || *end || v < INT_MIN || v > INT_MAX) {
    *rc = env_fail("%s=%s is not an integer", name, e);
    return 0;
  }
  *out = (int)v;
  return 1;
}
static int env_bool_strict(const char *name, int *out, int *rc) {
  const char *e = getenv(name);
  if (!e || !e[0]) return 0;
  if (strcmp(e, "0") && strcmp(e, "1")) {
    *rc = env_fail("%s must be 0 or 1", name);
    return 0;
  }
  *out = e[0] == '1';
  return 1;
}

int cwen_spec_from_env(cwen_spec_cfg *c) {
  if (!c) return host_fail(CWEN_EINVAL, "cwen_spec_from_env: cfg is NULL");
  int rc = 0, v;
  if (env_int_strict("CWEN_SPEC", &v, &rc)) {
    if (v != 0 && v != 1) return env_fail("CWEN_SPEC must be 0 or 1");
    c->spec = v;
  }
  if (env_int_strict("CWEN_SPEC_NGRAM_N", &v, &rc)) {
    if (v < 2 || v > 256) return env_fail("CWEN_SPEC_NGRAM_N must be in [2,256]");
    c->n_key = v;
  }
  if (env_int_strict("CWEN_SPEC_MAX_DRAFT", &v, &rc)) {
    if (v < 1 || v > 15) return env_fail("CWEN_SPEC_MAX_DRAFT must be in [1,15]");
    c->max_draft = v;
  }
  if (env_int_strict("CWEN_SPEC_MIN_DRAFT", &v, &rc)) {
    if (v < 1 || v > c->max_draft) return env_fail("CWEN_SPEC_MIN_DRAFT must be in [1,%d]", c->max_draft);
    c->min_draft = v;
  }
  if (env_int_strict("CWEN_SPEC_COOLDOWN", &v, &rc)) {
    if (v < 0 || v > 100000) return env_fail("CWEN_SPEC_COOLDOWN must be in [0,100000]");
    c->cooldown = v;
  }
  env_bool_strict("CWEN_SPEC_DEBUG", &c->debug, &rc);
  env_bool_strict("CWEN_MTP", &c->use_mtp, &rc);
  if (c->min_draft > c->max_draft)
    return env_fail("CWEN_SPEC_MIN_DRAFT (%d) exceeds CWEN_SPEC_MAX_DRAFT (%d)", c->min_draft, c->max_draft);
  return rc;
}

/* ---- n-gram drafter ---- */
int cwen_ngram_draft(const int32_t *h, int hn, int32_t *out, int n_key, int max_d) {
  if (!h || !out || n_key < 1 || hn <= n_key || max_d <= 0) return 0;
  const int32_t *tail = h + hn - n_key;
  int best = 0;
  /* newest match first; an older one wins only with a longer continuation */
  for (int j = hn - n_key - 1; j >= 0 && best < max_d; j--) {
    if (memcmp(h + j, tail, (size_t)n_key * sizeof(int32_t))) continue;
    int avail = hn - (j + n_key);
    if (avail > best) {
      int n = avail < max_d ? avail : max_d;
      memcpy(out, h + j + n_key, (size_t)n * sizeof(int32_t));
      best = n;
    }
  }
  return best;
}

/* Counted n-gram map: key of n_key ids -> (latest continuation, hit count),
   open addressing with linear probing, LFU eviction with backward-shift delete
   when full (run.c:4552-4654). */
#define NG_CAP ((size_t)1 << 18)
typedef struct {
  int32_t *keys, *tok, *cnt;
  unsigned char *used;
  size_t cap, used_n, hand;
  int nk;
} ngmap;

static uint64_t ng_hash(const int32_t *k, int n) {
  uint64_t h = 1469598103934665603ull;
  for (int i = 0; i < n; i++) {
    h ^= (uint64_t)(uint32_t)k[i];
    h *= 1099511628211ull;
    h ^= h >> 29;
  }
  return h;
}
static size_t ng_find(const ngmap *m, const int32_t *key, int *found) {
  size_t i = (size_t)ng_hash(key, m->nk) & (m->cap - 1);
  for (size_t p = 0; p < m->cap; p++, i = (i + 1) & (m->cap - 1)) {
    if (!m->used[i]) { *found = 0; return i; }
    if (!memcmp(m->keys + i * (size_t)m->nk, key, (size_t)m->nk * sizeof(int32_t))) { *found = 1; return i; }
  }
  *found = 0;
  return m->cap;
}
static void ng_evict_one(ngmap *m) {
  int mn = INT_MAX;
  for (size_t s = 0; s < m->cap; s++)
    if (m->used[s] && m->cnt[s] < mn) mn = m->cnt[s];
  size_t victim = m->cap;
  for (size_t k = 0; k < m->cap && victim == m->cap; k++) {
    size_t s = (m->hand + k) & (m->cap - 1);
    if (m->used[s] && m->cnt[s] == mn) victim = s;
  }
  if (victim == m->cap) return;
  m->hand = (victim + 1) & (m->cap - 1);
  size_t hole = victim;
  m->used[hole] = 0;
  for (size_t step = 1; step < m->cap; step++) {
    size_t j = (victim + step) & (m->cap - 1);
    if (!m->used[j]) break;
    size_t home = (size_t)ng_hash(m->keys + j * (size_t)m->nk, m->nk) & (m->cap - 1);
    size_t dh = (home - hole) & (m->cap - 1), dj = (j - hole) & (m->cap - 1);
    if (dh == 0 || dh > dj) {
      memcpy(m->keys + hole * (size_t)m->nk, m->keys + j * (size_t)m->nk, (size_t)m->nk * sizeof(int32_t));
      m->tok[hole] = m->tok[j];
      m->cnt[hole] = m->cnt[j];
      m->used[hole] = 1;
      m->used[j] = 0;
      hole = j;
    }
  }
  m->used_n--;
}
/* key -> tok with `hits` more hits (counts saturate at INT_MAX); a new key
   in a full map first evicts one least-hit entry. */
static void ng_update_n(ngmap *m, const int32_t *key, int32_t tok, int hits) {
  int found;
  size_t i = ng_find(m, key, &found);
  if (found) {
    m->cnt[i] = hits < INT_MAX - m->cnt[i] ? m->cnt[i] + hits : INT_MAX;
    m->tok[i] = tok;
    return;
  }
  if (i == m->cap) {
    ng_evict_one(m);
    i = ng_find(m, key, &found);
    if (i == m->cap) return;
  }
  memcpy(m->keys + i * (size_t)m->nk, key, (size_t)m->nk * sizeof(int32_t));
  m->tok[i] = tok;
  m->cnt[i] = hits;
  m->used[i] = 1;
  m->used_n++;
}
static void ng_update(ngmap *m, const int32_t *key, int32_t tok) { ng_update_n(m, key, tok, 1); }
static void ng_update_range(ngmap *m, const int32_t *h, int a, int b) {
  for (int p = a; p < b; p++)
    if (p - m->nk >= 0) ng_update(m, h + p - m->nk, h[p]);
}
static int ng_draft_map(const ngmap *m, const int32_t *h, int hn, int32_t *out, int max_d) {
  if (hn < m->nk || max_d <= 0) return 0;
  int32_t key[256];
  memcpy(key, h + hn - m->nk, (size_t)m->nk * sizeof(int32_t));
  int n = 0;
  while (n < max_d) {
    int found;
    size_t i = ng_find(m, key, &found);
    if (!found) break;
    out[n] = m->tok[i];
    memmove(key, key + 1, (size_t)(m->nk - 1) * sizeof(int32_t));
    key[m->nk - 1] = out[n];
    n++;
  }
  return n;
}
/* The n-gram proposal of a speculative cycle (run.c:4925-4933): chained
   map lookups from the tail key, replaced by the history scan when the scan
   proposes a longer run.  cap <= NG_MAX_PROPOSE. */
#define NG_MAX_PROPOSE 256
static int ng_propose(const ngmap *m, const int32_t *h, int hn, int32_t *out, int cap) {
  int32_t scan[NG_MAX_PROPOSE];
  int E = ng_draft_map(m, h, hn, out, cap);
  int esc = cwen_ngram_draft(h, hn, scan, m->nk, cap);
  if (esc > E) {
    E = esc;
    memcpy(out, scan, (size_t)E * sizeof(int32_t));
  }
  return E;
}
static int ng_init(ngmap *m, int nk) {
  memset(m, 0, sizeof *m);
  m->cap = NG_CAP;
  m->nk = nk;
  m->keys = (int32_t *)malloc(sizeof(int32_t) * NG_CAP * (size_t)nk);
  m->tok = (int32_t *)malloc(sizeof(int32_t) * NG_CAP);
  m->cnt = (int32_t *)calloc(NG_CAP, sizeof(int32_t));
  m->used = (unsigned char *)calloc(NG_CAP, 1);
  return (m->keys && m->tok && m->cnt && m->used) ? 0 : -1;
}
static void ng_free(ngmap *m) {
  free(m->keys);
  free(m->tok);
  free(m->cnt);
  free(m->used);
}

/* ---- NGC2 persistence of the map (run.c:4656-4716) ----
   Header {magic "NGC2", n_key, n_vocab, entries} (uint32), then per occupied
   slot in slot order {key[n_key], tok, cnt} (int32).  Loading merges counts
   into the live map; a missing, foreign (other n_key or vocabulary), damaged
   or truncated file contributes what it validly holds and never fails the
   run: the map only proposes drafts, which are verified anyway. */
#define NG_MAGIC 0x3243474eu

static int ng_save_file(const ngmap *m, const char *path, int vocab) {
  char tmp[4096];
  if (snprintf(tmp, sizeof tmp, "%s.tmp", path) >= (int)sizeof tmp)
    return host_fail(CWEN_EINVAL, "ngram cache: path too long");
  FILE *f = fopen(tmp, "wb");
  if (!f) return host_fail(CWEN_EINVAL, "ngram cache: %s: %s", tmp, strerror(errno));
  const uint32_t hdr[4] = {NG_MAGIC, (uint32_t)m->nk, (uint32_t)vocab, (uint32_t)m->used_n};
  int bad = fwrite(hdr, 4, 4, f) != 4;
  for (size_t i = 0; !bad && i < m->cap; i++) {
    if (!m->used[i]) continue;
    bad |= fwrite(m->keys + i * (size_t)m->nk, 4, (size_t)m->nk, f) != (size_t)m->nk;
    bad |= fwrite(&m->tok[i], 4, 1, f) != 1 || fwrite(&m->cnt[i], 4, 1, f) != 1;
  }
  bad |= fclose(f) != 0;
  if (bad) {
    remove(tmp);
    return host_fail(CWEN_EINVAL, "ngram cache: %s: write failed", tmp);
  }
  if (rename(tmp, path)) {
    remove(tmp);
    return host_fail(CWEN_EINVAL, "ngram cache: %s: %s", path, strerror(errno));
  }
  return CWEN_OK;
}

static int ng_load_file(ngmap *m, const char *path, int vocab) {
  FILE *f = fopen(path, "rb");
  if (!f) return 0;  /* no file yet: a cold start */
  uint32_t hdr[4];
  int n = 0;
  if (fread(hdr, 4, 4, f) == 4 && hdr[0] == NG_MAGIC && (int)hdr[1] == m->nk && (int)hdr[2] == vocab) {
    int32_t key[256], tc[2];
    for (uint32_t i = 0; i < hdr[3] && m->used_n < m->cap; i++) {
      if (fread(key, 4, (size_t)m->nk, f) != (size_t)m->nk || fread(tc, 4, 2, f) != 2) break;
      if (tc[0] < 0 || tc[0] >= vocab || tc[1] < 1) continue;
      ng_update_n(m, key, tc[0], tc[1]);
      n++;
    }
  } else {
    fprintf(stderr, "cwen: ngram cache %s: not an NGC2 map of this n_key and vocabulary; ignoring\n", path);
  }
  fclose(f);
  return n;
}

/* ---- the counted map as a drafter object (include/cwen_host.h) ---- */
struct cwen_ngram_map {
  ngmap m;
};

cwen_ngram_map *cwen_ngram_map_new(int n_key) {
  if (n_key < 2 || n_key > 256) {
    host_fail(CWEN_EINVAL, "cwen_ngram_map_new: n_key must be in [2,256]");
    return NULL;
  }
  cwen_ngram_map *p = (cwen_ngram_map *)malloc(sizeof *p);
  if (!p || ng_init(&p->m, n_key)) {
    if (p) ng_free(&p->m);
    free(p);
    host_fail(CWEN_ENOMEM, "cwen_ngram_map_new: out of host memory");
    return NULL;
  }
  return p;
}

void cwen_ngram_map_free(cwen_ngram_map *p) {
  if (!p) return;
  ng_free(&p->m);
  free(p);
}

void cwen_ngram_map_update(cwen_ngram_map *p, const int32_t *hist, int a, int b) {
  if (p && hist && a >= 0 && b > a) ng_update_range(&p->m, hist, a, b);
}

int cwen_ngram_map_save(const cwen_ngram_map *p, const char *path, int n_vocab) {
  if (!p || !path || !path[0] || n_vocab < 1) return host_fail(CWEN_EINVAL, "cwen_ngram_map_save: bad arguments");
  return ng_save_file(&p->m, path, n_vocab);
}

int cwen_ngram_map_load(cwen_ngram_map *p, const char *path, int n_vocab) {
  if (!p || !path || !path[0] || n_vocab < 1) return host_fail(CWEN_EINVAL, "cwen_ngram_map_load: bad arguments");
  return ng_load_file(&p->m, path, n_vocab);
}

int cwen_ngram_map_draft(const cwen_ngram_map *p, const int32_t *hist, int hn, int32_t *out, int max_d) {
  if (!p || !hist || !out || hn < 0) return host_fail(CWEN_EINVAL, "cwen_ngram_map_draft: bad arguments");
  if (max_d > NG_MAX_PROPOSE) max_d = NG_MAX_PROPOSE;
  return ng_propose(&p->m, hist, hn, out, max_d);
}

/* ---- drivers ---- */
#define BMAX 16
#define PF_ROWS 16

/* Prefill: slot 0 alone, then batched chunks; the last chunk's last row gets
   logits.  Returns the argmax after the prompt in *first. */
/* Fold committed slots pos0..pos0+n-1 (tokens t[0..n), rows 0..n-1 of the
   last forward) into the MTP stream (mtp_commit per committed position,
   run.c:4830-4849, 4948, 4987-4994). */
static int mtp_fold(int use_mtp, int pos0, const int32_t *t, int n) {
  if (!use_mtp) return 0;
  return cwen_cuda_mtp_commit_block(pos0, (const int *)t, n);
}

static int prefill(const int32_t *tokens, int n_tok, int *first, int use_mtp) {
  int rc = cwen_cuda_reset();
  if (rc) return rc;
  int i = 0;
  while (i < n_tok) {
    int B = n_tok - i < PF_ROWS ? n_tok - i : PF_ROWS;
    const int last = i + B == n_tok;
    rc = cwen_cuda_forward_block((const int *)tokens + i, B, last ? -1 : 0);
    if (rc) return rc;
    if (last) {
      rc = cwen_cuda_accept(NULL, first, NULL);
      if (rc) return rc;
    }
    rc = cwen_cuda_commit(B - 1);
    if (rc) return rc;
    rc = mtp_fold(use_mtp, i, tokens + i, B);
    if (rc) return rc;
    i += B;
  }
  return 0;
}

int cwen_generate(const int32_t *tokens, int n_tok, int n_gen, int32_t *out, const cwen_spec_cfg *cfg,
                  cwen_spec_stats *stats) {
  cwen_spec_stats st;
  memset(&st, 0, sizeof st);
  cwen_spec_cfg def;
  if (!cfg) {
    cwen_spec_defaults(&def);
    cfg = &def;
  }
  if (n_tok < 1 || n_gen < 0 || !tokens || (!out && n_gen))
    return host_fail(CWEN_EINVAL, "cwen_generate: need tokens, n_tok >= 1, n_gen >= 0 and out for n_gen ids");
  /* the knob ranges of spec_config_init (run.c:4021-4053): the driver's
     block buffers hold 1 + max_draft rows */
  if (cfg->max_draft < 1 || cfg->max_draft > BMAX - 1 || cfg->min_draft < 1 || cfg->n_key < 2 ||
      cfg->n_key > 256 || cfg->cooldown < 0 || cfg->cooldown > 100000)
    return host_fail(CWEN_EINVAL, "cwen_generate: spec knobs out of range (max_draft 1..%d, min_draft >= 1, "
                     "n_key 2..256, cooldown 0..100000)", BMAX - 1);
  /* the MTP head drafts only in speculative mode (run.c:5195) */
  const int use_mtp = cfg->spec && cfg->use_mtp && cwen_cuda_mtp_ready();
  int pend = 0, rc = prefill(tokens, n_tok, &pend, use_mtp);
  if (rc) return rc;
  const int ctx = cwen_cuda_ctx();
  int n = 0;
  if (!cfg->spec) {
    /* serial greedy decode (generate_tokens) */
    for (int g = 0; g < n_gen; g++) {
      if (cwen_cuda_n_past() >= ctx) break;
      out[n++] = pend;
      if (g + 1 == n_gen) break;
      int next = 0;
      rc = cwen_cuda_forward_serial(pend, 1, &next);
      if (rc) return rc;
      pend = next;
      st.plain_steps++;
    }
    if (stats) *stats = st;
    if (n < n_gen) fprintf(stderr, "cwen: context window full (ctx=%d); emitted %d of %d requested tokens\n", ctx, n, n_gen);
    return n;
  }
  /* block speculation (generate_tokens_spec) */
  int32_t *hist = (int32_t *)malloc(sizeof(int32_t) * ((size_t)n_tok + (size_t)n_gen + BMAX + 1));
  if (!hist) return CWEN_ENOMEM;
  memcpy(hist, tokens, (size_t)n_tok * sizeof(int32_t));
  int hn = n_tok, upd = 0, g = 0;
  ngmap ngm;
  const int use_map = !ng_init(&ngm, cfg->n_key);
  /* CWEN_NGRAM_CACHE: the map persists across runs (run.c:5198-5205) */
  const char *ngc = getenv("CWEN_NGRAM_CACHE");
  cwen_dims md;
  const int vocab = cwen_cuda_model_dims(&md) ? 0 : md.n_vocab;
  const int use_cache = use_map && ngc && ngc[0] && vocab > 0;
  if (use_cache) {
    const int got = ng_load_file(&ngm, ngc, vocab);
    if (got) fprintf(stderr, "ngram cache: loaded %d entries from %s\n", got, ngc);
  }
  if (n_gen > 0 && cwen_cuda_n_past() < ctx) {
    hist[hn++] = pend;
    out[n++] = pend;
    g = 1;
  }
  if (use_map) { ng_update_range(&ngm, hist, upd, hn); upd = hn; }
  const int cap_hard = cfg->max_draft;
  int E_cap = cap_hard, streak = 0, cool = 0, fa_streak = 0;
  int32_t blk[BMAX];
  int am[BMAX];
  while (g < n_gen) {
    const int n_past = cwen_cuda_n_past();
    if (n_past >= ctx) break;
    int E = 0;
    if (cool > 0) {
      cool--;
    } else {
      const int room = ctx - 1 - n_past;
      int cap = E_cap < room ? E_cap : room;
      if (cap > 0 && use_mtp) {
        E = cwen_cuda_mtp_draft(hist[hn - 1], blk + 1, cap);
        if (E < 0) { rc = E; goto fail; }
      } else if (cap > 0) {
        if (use_map) {
          E = ng_propose(&ngm, hist, hn, blk + 1, cap);
        } else {
          E = cwen_ngram_draft(hist, hn, blk + 1, cfg->n_key, cap);
        }
      }
      if (E && E < cfg->min_draft) E = 0;
    }
    blk[0] = hist[hn - 1];
    if (cfg->debug)
      fprintf(stderr, "spec dbg: cyc=%lld hn=%d n_past=%d E=%d tail0=%d\n", st.cycles, hn, n_past, E, hist[hn - 1]);
    int k = 0, ustar = 0;
    st.cycles++;
    if (E == 0) {
      rc = cwen_cuda_forward_serial(blk[0], 1, &ustar);
      if (rc) goto fail;
      rc = mtp_fold(use_mtp, n_past, blk, 1);
      if (rc) goto fail;
      st.plain_steps++;
    } else {
      const int B = E + 1;
      st.drafted++;
      rc = cwen_cuda_forward_block((const int *)blk, B, B);
      if (rc) goto fail;
      rc = cwen_cuda_accept(&k, &ustar, am);
      if (rc) goto fail;
      st.kept += k;
      if (k == E) st.full++;
      else st.shortw++;
      if (k == E) {
        if (++fa_streak >= 4 && E_cap < cap_hard) { E_cap++; fa_streak = 0; }
      } else {
        fa_streak = 0;
        E_cap = k > cfg->min_draft ? k : cfg->min_draft;
      }
      rc = cwen_cuda_commit(k);
      if (rc) goto fail;
      /* rows 0..k became context; the verify rows are the rows a re-score
         of pend + the kept drafts would give (batch invariance) */
      rc = mtp_fold(use_mtp, n_past, blk, k + 1);
      if (rc) goto fail;
    }
    for (int i = 0; i < k; i++) hist[hn++] = blk[i + 1];
    hist[hn++] = ustar;
    if (use_map) { ng_update_range(&ngm, hist, upd, hn); upd = hn; }
    for (int i = 0; i < k && g < n_gen; i++) { out[n++] = blk[i + 1]; g++; }
    if (g >= n_gen) break;
    out[n++] = ustar;
    g++;
    if (k == E) streak = 0;
    else if (++streak >= 3) { streak = 0; cool = cfg->cooldown; }
  }
  if (n < n_gen) fprintf(stderr, "cwen: context window full (ctx=%d); emitted %d of %d requested tokens\n", ctx, n, n_gen);
  fprintf(stderr, "spec: %lld cycles (%lld drafted, %lld full accept, %lld short; avg kept %.2f)\n", st.cycles,
          st.drafted, st.full, st.shortw, st.drafted ? (double)st.kept / (double)st.drafted : 0.0);
  if (use_cache && ngm.used_n && ng_save_file(&ngm, ngc, vocab))
    fprintf(stderr, "cwen: %s\n", cwen_cuda_last_error());  /* the run's tokens stand */
  if (use_map) ng_free(&ngm);
  free(hist);
  if (stats) *stats = st;
  return n;
fail:
  if (use_map) ng_free(&ngm);
  free(hist);
  return rc;
}
