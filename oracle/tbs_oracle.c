/*
 * TEST INFRASTRUCTURE ONLY - not part of the product.  See tbs_oracle.h.
 *
 * Plain C restatement of the reference FlashTrie GPU search semantics:
 *   - trie file parsing            lib/marisa/grimoire/trie/louds-trie.cc:722-746,
 *                                  vector/vector.h:448-457, bit-vector.h:201-217,
 *                                  flat-vector.h:154-173, tail.cc:311-314
 *   - rank1 / select0              vector/bit-vector.cc:398-498
 *   - child range + degree         tbs-kernels.cu:212-220 (select0 + next 0 bit)
 *   - label / link offset          louds-trie.cc:1036-1053
 *   - tail next_token              tail.cc:89-98
 *   - expansion of a branch parent tbs-kernels.cu:210-322
 *   - expansion of an in-link one  tbs-kernels.cu:324-371
 *   - step loop / early exit       tbs-kernels.cu:491-587
 *   - beam score / logp_norm       beam-state.h:13-26
 */
#include "tbs_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define TAIL_TERMINAL 0xFFFFFFFFu
#define REF_BLOCK 512 /* threads per CTA of the reference kernel (tbs-kernels.cu:10) */

typedef struct {
  uint64_t *units;
  uint64_t n_units;
  uint64_t size;
  uint64_t num_1s;
  uint32_t *ranks; /* 3 u32 per entry: abs, rel_lo, rel_hi */
  uint64_t n_ranks;
  uint32_t *select0s;
  uint64_t n_select0s;
} bits_t;

typedef struct {
  uint64_t *units;
  uint64_t n_units;
  uint32_t value_size;
  uint32_t mask;
  uint64_t size;
} flat_t;

struct oracle_trie {
  bits_t louds, terminal, link, end_flags;
  uint16_t *bases;
  uint64_t n_bases;
  flat_t extras, link_extras;
  uint32_t *tail;
  uint64_t n_tail;
  uint32_t flags;
  uint64_t num_nodes;
  void *file;
};

/* ------------------------------------------------------------ parsing */
typedef struct {
  const uint8_t *p;
  uint64_t left;
  int bad;
} cur_t;

static int need(cur_t *c, uint64_t n) {
  if (c->bad || n > c->left) {
    c->bad = 1;
    return 0;
  }
  return 1;
}
static uint64_t rd_u64(cur_t *c) {
  uint64_t v = 0;
  if (need(c, 8)) { memcpy(&v, c->p, 8); c->p += 8; c->left -= 8; }
  return v;
}
static uint32_t rd_u32(cur_t *c) {
  uint32_t v = 0;
  if (need(c, 4)) { memcpy(&v, c->p, 4); c->p += 4; c->left -= 4; }
  return v;
}
/* Vector<T>: u64 byte count, payload, zero padding to 8 (vector.h:448-457).
 * Points into the file buffer (kept alive by the trie). */
static const void *rd_vec(cur_t *c, uint64_t elem, uint64_t *count) {
  uint64_t bytes = rd_u64(c);
  const void *p;
  uint64_t pad;
  if (c->bad || bytes % elem) { c->bad = 1; *count = 0; return NULL; }
  if (!need(c, bytes)) { *count = 0; return NULL; }
  p = c->p;
  c->p += bytes;
  c->left -= bytes;
  pad = (8 - bytes % 8) % 8;
  if (need(c, pad)) { c->p += pad; c->left -= pad; }
  *count = bytes / elem;
  return p;
}
static void rd_bits(cur_t *c, bits_t *b) {
  uint64_t n1;
  b->units = (uint64_t *)rd_vec(c, 8, &b->n_units);
  b->size = rd_u32(c);
  b->num_1s = rd_u32(c);
  b->ranks = (uint32_t *)rd_vec(c, 12, &b->n_ranks);
  b->select0s = (uint32_t *)rd_vec(c, 4, &b->n_select0s);
  rd_vec(c, 4, &n1); /* select1s: not used by the search */
  if (b->num_1s > b->size || b->n_units * 64 < b->size) c->bad = 1;
}
static void rd_flat(cur_t *c, flat_t *f) {
  f->units = (uint64_t *)rd_vec(c, 8, &f->n_units);
  f->value_size = rd_u32(c);
  f->mask = rd_u32(c);
  f->size = rd_u64(c);
  if (f->value_size > 32 || (f->value_size && f->size > f->n_units * 64 / f->value_size)) c->bad = 1;
}

int oracle_load(const char *path, oracle_trie **out, char *err, int errlen) {
  FILE *fp = fopen(path, "rb");
  long n;
  uint8_t *buf;
  oracle_trie *t;
  cur_t c;
  uint64_t n_cache;
  *out = NULL;
  if (!fp) { snprintf(err, errlen, "cannot open %s", path); return -1; }
  fseek(fp, 0, SEEK_END);
  n = ftell(fp);
  fseek(fp, 0, SEEK_SET);
  buf = (uint8_t *)malloc((size_t)n + 8);
  if (!buf || fread(buf, 1, (size_t)n, fp) != (size_t)n) {
    fclose(fp);
    free(buf);
    snprintf(err, errlen, "cannot read %s", path);
    return -1;
  }
  fclose(fp);
  t = (oracle_trie *)calloc(1, sizeof(*t));
  t->file = buf;
  c.p = buf;
  c.left = (uint64_t)n;
  c.bad = 0;
  if (n < 16 || memcmp(buf, "We love Marisa.", 16) != 0) {
    snprintf(err, errlen, "bad header");
    oracle_free(t);
    return -2;
  }
  c.p += 16;
  c.left -= 16;
  rd_bits(&c, &t->louds);
  rd_bits(&c, &t->terminal);
  rd_bits(&c, &t->link);
  t->bases = (uint16_t *)rd_vec(&c, 2, &t->n_bases);
  rd_flat(&c, &t->extras);
  rd_flat(&c, &t->link_extras);
  t->tail = (uint32_t *)rd_vec(&c, 4, &t->n_tail);
  rd_bits(&c, &t->end_flags);
  if (!c.bad && t->link.num_1s != 0 && t->n_tail == 0) {
    snprintf(err, errlen, "multi-trie files are not supported by the search");
    oracle_free(t);
    return -3;
  }
  rd_vec(&c, 12, &n_cache);
  rd_u32(&c);
  t->flags = rd_u32(&c);
  if (c.bad) {
    snprintf(err, errlen, "truncated or malformed trie");
    oracle_free(t);
    return -2;
  }
  t->num_nodes = t->louds.size / 2 - 1;
  *out = t;
  return 0;
}

void oracle_free(oracle_trie *t) {
  if (!t) return;
  free(t->file);
  free(t);
}
uint64_t oracle_num_nodes(const oracle_trie *t) { return t->num_nodes; }
uint64_t oracle_num_keys(const oracle_trie *t) { return t->terminal.num_1s; }

/* ---------------------------------------------------------- bit ops */
static int bit_get(const bits_t *b, uint64_t i) { return (int)((b->units[i >> 6] >> (i & 63)) & 1u); }

static uint32_t rank_rel(const uint32_t *r, int k) {
  /* rank-index.h:287-307 */
  switch (k) {
    case 1: return r[1] & 0x7Fu;
    case 2: return (r[1] >> 7) & 0xFFu;
    case 3: return (r[1] >> 15) & 0xFFu;
    case 4: return (r[1] >> 23) & 0x1FFu;
    case 5: return r[2] & 0x1FFu;
    case 6: return (r[2] >> 9) & 0x1FFu;
    case 7: return (r[2] >> 18) & 0x1FFu;
  }
  return 0;
}

/* bit-vector.cc:398-436 */
static uint64_t rank1(const bits_t *b, uint64_t i) {
  const uint32_t *r = b->ranks + 3 * (i / 512);
  uint64_t off = r[0] + rank_rel(r, (int)((i / 64) % 8));
  uint64_t m = (i % 64) ? ((1ull << (i % 64)) - 1) : 0;
  return off + (uint64_t)__builtin_popcountll(b->units[i / 64] & m);
}

/* i-th set bit of `w` (ith_set_pos, bit-vector.cc:11-16) */
static uint64_t ith_set(uint64_t w, uint64_t i) {
  uint64_t k;
  for (k = 0; k < i; k++) w &= w - 1;
  return (uint64_t)__builtin_ctzll(w);
}

/* bit-vector.cc:438-498: select sample, then a linear (<= 10 blocks) or
 * binary search over the rank blocks, then the sub-block and bit. */
static uint64_t select0(const bits_t *b, uint64_t i) {
  uint64_t sid = i / 512, begin, end, rid, unit;
  const uint32_t *r;
  if (i % 512 == 0) return b->select0s[sid];
  begin = b->select0s[sid] / 512;
  end = (b->select0s[sid + 1] + 511) / 512;
  if (begin + 10 >= end) {
    while (i >= (begin + 1) * 512 - b->ranks[3 * (begin + 1)]) ++begin;
  } else {
    while (begin + 1 < end) {
      uint64_t mid = (begin + end) / 2;
      if (i < mid * 512 - b->ranks[3 * mid]) end = mid; else begin = mid;
    }
  }
  rid = begin;
  i -= rid * 512 - b->ranks[3 * rid];
  r = b->ranks + 3 * rid;
  unit = rid * 8;
  /* zeros before sub-block k of the block = 64k - rel_k */
  {
    int k;
    for (k = 7; k >= 1; k--) {
      uint64_t zeros_before = 64ull * (uint64_t)k - rank_rel(r, k);
      if (i >= zeros_before) {
        unit += (uint64_t)k;
        i -= zeros_before;
        break;
      }
    }
  }
  return unit * 64 + ith_set(~b->units[unit], i);
}

/* First 0 bit at or after position i (warp_find_next_unset, bit-vector.h:86-113). */
static uint64_t next_zero(const bits_t *b, uint64_t i) {
  uint64_t w = b->units[i / 64] | ~(~0ull << (i % 64));
  uint64_t u = i / 64;
  while (~w == 0) w = b->units[++u];
  return u * 64 + (uint64_t)__builtin_ctzll(~w);
}

static uint32_t flat_get(const flat_t *f, uint64_t i) {
  uint64_t pos = i * f->value_size, u = pos / 64, off = pos % 64;
  if (off + f->value_size <= 64) return (uint32_t)(f->units[u] >> off) & f->mask;
  return (uint32_t)((f->units[u] >> off) | (f->units[u + 1] << (64 - off))) & f->mask;
}

static uint32_t node_label(const oracle_trie *t, uint64_t n) { return (uint32_t)t->bases[n] | (flat_get(&t->extras, n) << 16); }
static uint64_t node_link(const oracle_trie *t, uint64_t n) {
  uint32_t hi = flat_get(&t->link_extras, rank1(&t->link, n));
  return (uint64_t)(uint32_t)((uint32_t)t->bases[n] | (hi << 16));
}
/* tail.cc:89-98: returns the token at *off, advances, sets *end */
static uint32_t tail_next(const oracle_trie *t, uint64_t *off, int *end) {
  uint32_t tok = t->tail[(*off)++];
  if (t->end_flags.size == 0) *end = t->tail[*off] == TAIL_TERMINAL;
  else *end = bit_get(&t->end_flags, *off - 1);
  return tok;
}

/* Node reached by `key` (reference LoudsTrie::find_child, louds-trie.cc:764-808,
 * with a text/binary tail match), or -1. */
static int64_t walk(const oracle_trie *t, const uint32_t *key, uint32_t len) {
  uint64_t node = 0;
  uint32_t pos = 0;
  while (pos < len) {
    uint64_t lp = select0(&t->louds, node) + 1;
    uint64_t child;
    int found = 0;
    if (!bit_get(&t->louds, lp)) return -1;
    child = lp - node - 1;
    for (; bit_get(&t->louds, lp); ++lp, ++child) {
      if (bit_get(&t->link, child)) {
        uint64_t off = node_link(t, child);
        if (t->tail[off] != key[pos]) continue;
        for (;;) {
          int end;
          uint32_t tok = tail_next(t, &off, &end);
          if (pos >= len || tok != key[pos]) return -1;
          pos++;
          if (end) break;
        }
        found = 1;
        break;
      } else if (node_label(t, child) == key[pos]) {
        pos++;
        found = 1;
        break;
      }
    }
    if (!found) return -1;
    node = child;
  }
  return (int64_t)node;
}

int oracle_lookup(const oracle_trie *t, const uint32_t *key, uint32_t len) {
  const int64_t node = walk(t, key, len);
  return node >= 0 && bit_get(&t->terminal, (uint64_t)node);
}

/* Key id of `key`: the rank of its terminal node among the terminal nodes
 * (reference LoudsTrie::lookup, louds-trie.cc:56-72), or -1. */
int64_t oracle_lookup_id(const oracle_trie *t, const uint32_t *key, uint32_t len) {
  const int64_t node = walk(t, key, len);
  if (node < 0 || !bit_get(&t->terminal, (uint64_t)node)) return -1;
  return (int64_t)rank1(&t->terminal, (uint64_t)node);
}

/* ------------------------------------------------------------ search */
typedef struct {
  int64_t parent; /* arena index of the parent beam, -1 for the root */
  uint32_t token;
  uint32_t depth;
} hist_t;

typedef struct {
  double lpn;
  double score;
  uint32_t node;
  uint32_t depth;
  uint64_t off;   /* next tail cell for an in-link beam */
  int in_link;
  int64_t hist;   /* arena index of this beam's (parent, token) record */
} beam_t;

/* Monotone map of a double onto u64 (-0.0 folded onto +0.0), so the order is
 * total even for NaN inputs. */
static uint64_t ord(double d) {
  uint64_t u;
  memcpy(&u, &d, 8);
  if ((u << 1) == 0) u = 0;
  return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

/* "a ranks above b" in the pinned order */
static int better(const beam_t *a, const beam_t *b) {
  if (ord(a->lpn) != ord(b->lpn)) return ord(a->lpn) > ord(b->lpn);
  if (a->node != b->node) return a->node > b->node;
  if (a->depth != b->depth) return a->depth > b->depth;
  return ord(a->score) > ord(b->score);
}
static int cmp_desc(const void *x, const void *y) {
  const beam_t *a = (const beam_t *)x, *b = (const beam_t *)y;
  if (better(a, b)) return -1;
  if (better(b, a)) return 1;
  return 0;
}

typedef struct {
  beam_t *v;
  uint64_t n, cap;
} bvec_t;
static int bpush(bvec_t *b, const beam_t *x) {
  if (b->n == b->cap) {
    uint64_t nc = b->cap ? 2 * b->cap : 64;
    beam_t *nv = (beam_t *)realloc(b->v, nc * sizeof(beam_t));
    if (!nv) return -1;
    b->v = nv;
    b->cap = nc;
  }
  b->v[b->n++] = *x;
  return 0;
}
typedef struct {
  hist_t *v;
  uint64_t n, cap;
} hvec_t;
static int64_t hpush(hvec_t *h, int64_t parent, uint32_t token, uint32_t depth) {
  if (h->n == h->cap) {
    uint64_t nc = h->cap ? 2 * h->cap : 256;
    hist_t *nv = (hist_t *)realloc(h->v, nc * sizeof(hist_t));
    if (!nv) return -2;
    h->v = nv;
    h->cap = nc;
  }
  h->v[h->n].parent = parent;
  h->v[h->n].token = token;
  h->v[h->n].depth = depth;
  return (int64_t)h->n++;
}

/* keep the best k of b (in place); returns 1 when the cut separates two
 * candidates of equal logp_norm */
static int keep_top(bvec_t *b, uint64_t k) {
  int tie;
  if (b->n <= k) return 0;
  qsort(b->v, b->n, sizeof(beam_t), cmp_desc);
  tie = k > 0 && ord(b->v[k - 1].lpn) == ord(b->v[k].lpn);
  b->n = k;
  return tie;
}

static uint64_t ceil_log2(uint64_t x) {
  uint64_t r = 0;
  while ((1ull << r) < x) r++;
  return r;
}

int oracle_tbs(const oracle_trie *t, uint32_t L, uint32_t K, const uint32_t *beams,
               const uint32_t *topk_id, const float *topk_logp, float token_logp_threshold,
               double sent_logp_threshold, double length_norm, int early_exit, uint32_t out_cap,
               uint32_t out_stride, uint32_t *out_n, double *out_lpn, uint32_t *out_len,
               uint32_t *out_tok, oracle_stats *stats) {
  const double tt = (double)token_logp_threshold;
  const double st = sent_logp_threshold;
  uint32_t final_beam, step, i;
  double *factor;
  bvec_t cur = {0}, next = {0}, sel = {0};
  hvec_t hist = {0};
  uint64_t sel_pushes = 0, bytes = 0;
  uint32_t ties = 0;
  int rc = 0;
  beam_t root;

  *out_n = 0;
  if (stats) memset(stats, 0, sizeof(*stats));
  if (L == 0) return -1;
  final_beam = beams[L - 1];
  if (final_beam == 0) return 0; /* tbs-kernels.cu:675-678 */
  if (out_cap < final_beam || out_stride < L) return -2;
  if (t->flags & 0x20000u) return -1; /* weight order: children not label-sorted */

  /* logp_norm = score * (6/(5+depth))^length_norm (beam-state.h:24-26) */
  factor = (double *)malloc(sizeof(double) * (L + 1));
  for (i = 0; i <= L; i++) factor[i] = pow(6.0 / (5.0 + (double)i), length_norm);

  memset(&root, 0, sizeof(root));
  root.hist = -1;
  root.lpn = 0.0 * factor[0];
  if (bpush(&cur, &root)) { rc = -3; goto done; }

  for (step = 0; step < L; step++) {
    const uint32_t *row = topk_id + (uint64_t)step * K;
    const float *lp = topk_logp + (uint64_t)step * K;
    uint64_t p, np_in = 0, np_br = 0, deg_sum = 0, nx = 0, ns = 0;
    if (cur.n == 0 || (early_exit && sel_pushes >= final_beam)) break;
    next.n = 0;
    bytes += (uint64_t)K * 8; /* the row: ids + logp */
    for (p = 0; p < cur.n; p++) {
      const beam_t par = cur.v[p];
      if (par.in_link) {
        /* tbs-kernels.cu:324-371: the next tail token must appear in the row;
         * each of the reference's REF_BLOCK threads takes its first match. */
        uint64_t off = par.off;
        int end;
        uint32_t tok = tail_next(t, &off, &end);
        uint32_t r;
        np_in++;
        bytes += 32;
        for (r = 0; r < REF_BLOCK && r < K; r++) {
          uint32_t j;
          for (j = r; j < K; j += REF_BLOCK) {
            if (row[j] != tok) continue;
            if ((double)lp[j] <= tt || par.score + (double)lp[j] <= st) break;
            {
              beam_t ch = par;
              ch.score = par.score + (double)lp[j];
              ch.depth = par.depth + 1;
              ch.lpn = ch.score * factor[ch.depth];
              ch.off = off;
              ch.hist = hpush(&hist, par.hist, tok, ch.depth);
              if (ch.hist < 0) { rc = -3; goto done; }
              if (end) {
                bytes += 32; /* terminal flag */
                if (bit_get(&t->terminal, ch.node)) {
                  if (bpush(&sel, &ch)) { rc = -3; goto done; }
                  ns++;
                }
              } else {
                if (bpush(&next, &ch)) { rc = -3; goto done; }
                nx++;
              }
            }
            break;
          }
        }
      } else {
        /* tbs-kernels.cu:210-322: per proposal, binary search the children
         * by first label (a link child's first label is its first tail token). */
        const uint64_t base = select0(&t->louds, par.node) + 1;
        const uint64_t first = base - par.node - 1;
        const uint64_t deg = next_zero(&t->louds, base) - base;
        uint32_t j;
        np_br++;
        deg_sum += deg;
        bytes += 32; /* child range */
        if (deg == 0) continue;
        {
          uint64_t scan = (deg + 7) / 8 + 1, search = (uint64_t)K * (ceil_log2(deg + 1));
          bytes += 32 * (scan < search ? scan : search);
        }
        for (j = 0; j < K; j++) {
          int64_t lo = 0, hi = (int64_t)deg - 1;
          uint64_t c = 0, loff = 0;
          int is_link = 0, end = 0, hit = 0;
          if ((double)lp[j] <= tt || par.score + (double)lp[j] <= st) continue;
          while (lo <= hi) {
            int64_t mid = (lo + hi) >> 1;
            uint32_t lab;
            c = first + (uint64_t)mid;
            is_link = bit_get(&t->link, c);
            if (!is_link) {
              lab = node_label(t, c);
            } else {
              loff = node_link(t, c);
              lab = tail_next(t, &loff, &end);
            }
            if (lab == row[j]) { hit = 1; break; }
            if (lab < row[j]) lo = mid + 1; else hi = mid - 1;
          }
          if (!hit) continue;
          {
            beam_t ch;
            memset(&ch, 0, sizeof(ch));
            ch.node = (uint32_t)c;
            ch.score = par.score + (double)lp[j];
            ch.depth = par.depth + 1;
            ch.lpn = ch.score * factor[ch.depth];
            ch.hist = hpush(&hist, par.hist, row[j], ch.depth);
            if (ch.hist < 0) { rc = -3; goto done; }
            bytes += 32; /* child flags */
            if (!is_link) {
              if (bit_get(&t->terminal, c)) {
                if (bpush(&sel, &ch)) { rc = -3; goto done; }
                ns++;
              }
              if (bpush(&next, &ch)) { rc = -3; goto done; }
              nx++;
            } else {
              bytes += 64; /* link offset + next tail cells */
              ch.in_link = 1;
              ch.off = loff;
              if (end) {
                if (bit_get(&t->terminal, c)) {
                  if (bpush(&sel, &ch)) { rc = -3; goto done; }
                  ns++;
                }
              } else {
                if (bpush(&next, &ch)) { rc = -3; goto done; }
                nx++;
              }
            }
          }
        }
      }
    }
    bytes += 64 * (nx + ns); /* candidate write + read at selection */
    sel_pushes += ns;
    if (stats && step < ORACLE_MAX_STEPS) {
      stats->parents_inlink[step] = np_in;
      stats->parents_branch[step] = np_br;
      stats->degree_sum[step] = deg_sum;
      stats->next_pushes[step] = nx;
      stats->sel_pushes[step] = ns;
      stats->steps_run = step + 1;
    }
    ties += keep_top(&next, beams[step]);
    ties += keep_top(&sel, final_beam);
    {
      bvec_t tmp = cur;
      cur = next;
      next = tmp;
    }
  }

  ties += keep_top(&sel, final_beam);
  qsort(sel.v, sel.n, sizeof(beam_t), cmp_desc);
  /* ascending output: worst first (tbs-kernels.cu:415-421) */
  for (i = 0; i < sel.n; i++) {
    const beam_t *b = &sel.v[sel.n - 1 - i];
    int64_t h = b->hist;
    uint32_t d = b->depth;
    out_lpn[i] = b->lpn;
    out_len[i] = d;
    while (h >= 0 && d > 0) {
      out_tok[(uint64_t)i * out_stride + (--d)] = hist.v[h].token;
      h = hist.v[h].parent;
    }
    bytes += 12 + 4ull * b->depth;
  }
  *out_n = (uint32_t)sel.n;
  if (stats) {
    stats->bytes_alg = bytes;
    stats->ties_at_cut = ties;
  }

done:
  free(factor);
  free(cur.v);
  free(next.v);
  free(sel.v);
  free(hist.v);
  return rc;
}
