/*
 * CPU oracle for the DDTree verification hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C restatement of the reference
 * algorithms (ddtree.py of the DDTree research code) used as the checker for the
 * CUDA kernels.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load it.  The product path never calls into it.
 *
 * Parity pin: tests/test_oracle_golden.py checks every function below against the
 * golden vectors in tests/golden/, which tests/golden/make_golden.py produced by
 * running the reference's own Python functions.
 *
 * Conventions shared with the CUDA kernels (and written down here once):
 *   - log Z of a row is computed as  m + log(sum_i exp((double)x_i - (double)m))
 *     entirely in double and rounded once to float (m = row max).  torch's fp32
 *     logsumexp agrees with it to within a couple of float ulps.
 *   - top-k order is (value descending, index ascending): the canonical tie rule.
 *   - top log-prob = (float)(top_value - logZ) computed in float, as
 *     `top_logits - log_z` does in ddtree.py:109.
 *   - argmax ties go to the lowest index; a NaN counts as larger than any number
 *     (torch.argmax semantics).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_EINVAL -1
#define ORC_ENOMEM -2

/* ------------------------------------------------------------------------- */
/* per-depth log Z + top-k (ddtree.py:102-110)                                */
/* ------------------------------------------------------------------------- */

typedef struct {
  float v;
  int64_t i;
} orc_vi;

static int orc_vi_cmp(const void* a, const void* b) {
  const orc_vi* x = (const orc_vi*)a;
  const orc_vi* y = (const orc_vi*)b;
  if (x->v > y->v) return -1;
  if (x->v < y->v) return 1;
  return (x->i < y->i) ? -1 : (x->i > y->i);
}

/* logits: [L, V] float32 (bf16 callers widen exactly before calling).
 * Outputs: top_lp [L, k], top_ids [L, k], logz [L]. */
int orc_logz_topk(const float* logits, int64_t L, int64_t V, int64_t k, float* top_lp,
                  int64_t* top_ids, float* logz) {
  if (L < 0 || V <= 0 || k <= 0 || k > V) return ORC_EINVAL;
  orc_vi* buf = (orc_vi*)malloc(sizeof(orc_vi) * (size_t)V);
  if (!buf) return ORC_ENOMEM;
  for (int64_t d = 0; d < L; ++d) {
    const float* row = logits + d * V;
    float m = row[0];
    for (int64_t i = 1; i < V; ++i)
      if (row[i] > m) m = row[i];
    double s = 0.0;
    for (int64_t i = 0; i < V; ++i) s += exp((double)row[i] - (double)m);
    float lz = (float)((double)m + log(s));
    logz[d] = lz;
    for (int64_t i = 0; i < V; ++i) {
      buf[i].v = row[i];
      buf[i].i = i;
    }
    qsort(buf, (size_t)V, sizeof(orc_vi), orc_vi_cmp);
    for (int64_t j = 0; j < k; ++j) {
      top_lp[d * k + j] = buf[j].v - lz; /* float subtraction */
      top_ids[d * k + j] = buf[j].i;
    }
  }
  free(buf);
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* best-first tree (ddtree.py:116-147)                                        */
/* ------------------------------------------------------------------------- */

/* A heap item mirrors the reference tuple (-logw, ranks, parent, depth, rank, logw).
 * Rank tuples are unique per candidate, so the order (-logw, ranks) is total and
 * the pop sequence does not depend on how the priority queue is implemented. */
typedef struct {
  double neg_logw;
  double logw;
  int32_t parent;
  int32_t depth;
  int32_t rank;
  int32_t ranks_off; /* offset of this item's rank tuple in the rank pool */
} orc_item;

typedef struct {
  orc_item* items;
  int64_t n;
  const int32_t* pool;
} orc_heap;

static int orc_item_less(const orc_heap* h, const orc_item* a, const orc_item* b) {
  if (a->neg_logw < b->neg_logw) return 1;
  if (a->neg_logw > b->neg_logw) return 0;
  /* Python tuple order on the rank tuples: element-wise, shorter prefix first. */
  const int32_t* ra = h->pool + a->ranks_off;
  const int32_t* rb = h->pool + b->ranks_off;
  int32_t la = a->depth, lb = b->depth;
  int32_t n = la < lb ? la : lb;
  for (int32_t j = 0; j < n; ++j) {
    if (ra[j] < rb[j]) return 1;
    if (ra[j] > rb[j]) return 0;
  }
  if (la != lb) return la < lb;
  /* identical rank tuples never occur for distinct candidates; fall through. */
  if (a->parent != b->parent) return a->parent < b->parent;
  return 0;
}

static void orc_heap_push(orc_heap* h, orc_item it) {
  int64_t i = h->n++;
  h->items[i] = it;
  while (i > 0) {
    int64_t p = (i - 1) / 2;
    if (!orc_item_less(h, &h->items[i], &h->items[p])) break;
    orc_item t = h->items[i];
    h->items[i] = h->items[p];
    h->items[p] = t;
    i = p;
  }
}

static orc_item orc_heap_pop(orc_heap* h) {
  orc_item top = h->items[0];
  h->items[0] = h->items[--h->n];
  int64_t i = 0;
  for (;;) {
    int64_t l = 2 * i + 1, r = l + 1, m = i;
    if (l < h->n && orc_item_less(h, &h->items[l], &h->items[m])) m = l;
    if (r < h->n && orc_item_less(h, &h->items[r], &h->items[m])) m = r;
    if (m == i) break;
    orc_item t = h->items[i];
    h->items[i] = h->items[m];
    h->items[m] = t;
    i = m;
  }
  return top;
}

/* top_lp/top_ids: [L, k].  Outputs sized for `budget`:
 *   node_ids[budget], node_depths[budget], parents[budget + 1] (parents[0] = -1),
 *   *node_count.  Returns ORC_OK. */
int orc_build_tree(const float* top_lp, const int64_t* top_ids, int64_t L, int64_t k,
                   int64_t budget, int64_t* node_ids, int64_t* node_depths, int32_t* parents,
                   int64_t* node_count) {
  *node_count = 0;
  if (budget <= 0 || L <= 0) {
    parents[0] = -1;
    return ORC_OK;
  }
  if (k <= 0) return ORC_EINVAL;
  /* each pop pushes at most 2 items; each item owns a rank tuple of <= L ints. */
  int64_t max_items = 2 * budget + 2;
  orc_heap h;
  h.items = (orc_item*)malloc(sizeof(orc_item) * (size_t)max_items);
  int32_t* pool = (int32_t*)malloc(sizeof(int32_t) * (size_t)(max_items * L));
  if (!h.items || !pool) {
    free(h.items);
    free(pool);
    return ORC_ENOMEM;
  }
  h.n = 0;
  h.pool = pool;
  int64_t pool_used = 0;

  double first = (double)top_lp[0];
  orc_item it0 = {-first, first, 0, 1, 0, (int32_t)pool_used};
  pool[pool_used++] = 0;
  orc_heap_push(&h, it0);

  parents[0] = -1;
  int64_t count = 0;
  while (h.n > 0 && count < budget) {
    orc_item it = orc_heap_pop(&h);
    int64_t token = top_ids[(int64_t)(it.depth - 1) * k + it.rank];
    int64_t cur = count + 1;
    node_ids[count] = token;
    node_depths[count] = it.depth;
    parents[cur] = it.parent;
    count++;
    /* copy this item's rank tuple before pushing (the pool only grows). */
    int32_t off = it.ranks_off;
    if (it.rank + 1 < k) {
      double lp_cur = (double)top_lp[(int64_t)(it.depth - 1) * k + it.rank];
      double lp_nxt = (double)top_lp[(int64_t)(it.depth - 1) * k + it.rank + 1];
      double sib = it.logw - lp_cur + lp_nxt;
      orc_item s = {-sib, sib, it.parent, it.depth, it.rank + 1, (int32_t)pool_used};
      for (int32_t j = 0; j < it.depth - 1; ++j) pool[pool_used + j] = pool[off + j];
      pool[pool_used + it.depth - 1] = it.rank + 1;
      pool_used += it.depth;
      orc_heap_push(&h, s);
    }
    if (it.depth < L) {
      double child = it.logw + (double)top_lp[(int64_t)it.depth * k + 0];
      orc_item c = {-child, child, (int32_t)cur, it.depth + 1, 0, (int32_t)pool_used};
      for (int32_t j = 0; j < it.depth; ++j) pool[pool_used + j] = pool[off + j];
      pool[pool_used + it.depth] = 0;
      pool_used += it.depth + 1;
      orc_heap_push(&h, c);
    }
  }
  *node_count = count;
  free(h.items);
  free(pool);
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* visibility (ddtree.py:151-159) and ancestor bitmasks                       */
/* ------------------------------------------------------------------------- */

/* vis: [n, n] bytes, row i = ancestors-or-self of node i. */
int orc_visibility(const int32_t* parents, int64_t n, uint8_t* vis) {
  memset(vis, 0, (size_t)(n * n));
  if (n <= 0) return ORC_OK;
  vis[0] = 1;
  for (int64_t i = 1; i < n; ++i) {
    int32_t p = parents[i];
    if (p < 0 || p >= i) return ORC_EINVAL;
    memcpy(vis + i * n, vis + (int64_t)p * n, (size_t)i);
    vis[i * n + i] = 1;
  }
  return ORC_OK;
}

/* bits: [n, words] uint32, bit j of row i set iff node j is an ancestor-or-self of i. */
int orc_ancestor_bits(const int32_t* parents, int64_t n, int64_t words, uint32_t* bits) {
  if (words * 32 < n) return ORC_EINVAL;
  memset(bits, 0, sizeof(uint32_t) * (size_t)(n * words));
  for (int64_t i = 0; i < n; ++i) {
    int64_t j = i;
    while (j >= 0) {
      bits[i * words + j / 32] |= 1u << (j % 32);
      j = parents[j];
      if (j >= i) return ORC_EINVAL;
    }
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* greedy posterior + accept walk (model/utils.py:28-30, ddtree.py:270-281)   */
/* ------------------------------------------------------------------------- */

int orc_argmax(const float* x, int64_t rows, int64_t cols, int64_t* out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = x + r * cols;
    int64_t best = 0;
    float bv = row[0];
    for (int64_t c = 1; c < cols; ++c) {
      float v = row[c];
      if (isnan(bv)) break;
      if (isnan(v) || v > bv) {
        bv = v;
        best = c;
      }
    }
    out[r] = best;
  }
  return ORC_OK;
}

/* child_maps[p][token] = child, built from parents/node_ids (node i >= 1 has token
 * node_ids[i - 1]).  A later child with the same token under the same parent would
 * overwrite an earlier one in the reference dict; the walk below does the same by
 * keeping the last match. */
int orc_follow(const int32_t* parents, const int64_t* node_ids, int64_t n,
               const int64_t* posterior, int64_t* accepted, int64_t* n_accepted,
               int64_t* next_token) {
  int64_t cur = 0, cnt = 0;
  accepted[cnt++] = 0;
  int64_t tok = posterior[0];
  for (;;) {
    int64_t child = -1;
    for (int64_t i = 1; i < n; ++i)
      if (parents[i] == cur && node_ids[i - 1] == tok) child = i;
    if (child < 0) break;
    cur = child;
    accepted[cnt++] = cur;
    tok = posterior[cur];
  }
  *n_accepted = cnt;
  *next_token = tok;
  return ORC_OK;
}
