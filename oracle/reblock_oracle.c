/*
 * CPU restatement of the landmark-tree-v2 reblock permutation (the default "full" Spark
 * mode: cosine distance, one token per group, 32 midpoint landmarks, linear aggregation,
 * parent order, two mean-update proxy iterations from the farthest pair; any child count from
 * 2 to 64, so the power-of-two, arbitrary and power-of-two-arbitrary-final fanout modes all
 * run through it).  TEST INFRASTRUCTURE ONLY: the tests and the smoke check compare the CUDA
 * reblock against it; the product never links or calls it.
 *
 * Follows h3_sparse_attention:
 *   - remainder:   landmark_tree_clustering.py:56-82 (_largest_norm_remainder: the N mod 64
 *                  largest squared norms, equal norms to the lower index) and :85-146
 *                  (_initial_hilbert_partition: stable split of the root order)
 *   - recursion:   landmark_tree_v2.py:297-787 (_recursive_landmark_tree_v2, reference arm:
 *                  per node child capacities 64 x budget, children laid out in order)
 *   - landmarks:   landmark_tree_v2.py:175-228 (_torch_interval_landmarks, midpoint mode) with
 *                  landmark_tree_clustering.py:49-53 (_midpoint_positions)
 *   - proxy tree:  landmark_v2_cosine.py:40-84 (cosine_proxy_scores_reference) and, for any
 *                  child count, landmark_v2_terminal.py:62-148 (node_split_reference) over the
 *                  split topology of landmark_v2_terminal.py:11-33 (split_topology: a node of
 *                  children [s0, s1) splits at s0 + (s1 - s0 + 1) / 2, internal nodes numbered
 *                  breadth first, a child's landmark weights kept in slot 2 * node + 1 or + 2)
 *   - routing:     landmark_tree_clustering.py:290-515 (_exact_tree_route, CPU arm: per
 *                  internal node the left capacity goes to the smallest (score, index))
 *   - partition:   landmark_tree_clustering.py:516-565 (_stable_counting_partition)
 *
 * Canonical fp32 arithmetic, shared bit for bit with the CUDA kernels.  A D-vector is split
 * over 32 lanes, lane l holding the c = D/32 consecutive elements [l*c, l*c + c):
 *   dot(a, b):  lane partial p_l = a0*b0, then p_l = fma(a_i, b_i, p_l) for i = 1 .. c-1;
 *               then five butterfly rounds p_l <- p_l + p_(l xor o), o = 16, 8, 4, 2, 1.
 *   unit(x):    x_i / max(sqrt(dot(x, x)), 1e-12)       (IEEE division and square root)
 *   mean:       acc = 0; acc = fma(w_j, x_j, acc) for landmarks j = 0 .. 31; acc / capacity
 * Compile with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define RB_LANES 32
#define RB_MAX_D 256
#define RB_LANDMARKS 32
#define RB_MAX_CHILDREN 64

static float rb_bf16(uint16_t x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static float rb_dot(const float* a, const float* b, int d) {
  const int c = d / RB_LANES;
  float p[RB_LANES];
  for (int l = 0; l < RB_LANES; ++l) {
    const float* x = a + l * c;
    const float* y = b + l * c;
    float acc = x[0] * y[0];
    for (int i = 1; i < c; ++i) acc = fmaf(x[i], y[i], acc);
    p[l] = acc;
  }
  for (int o = 16; o >= 1; o >>= 1) {
    float q[RB_LANES];
    for (int l = 0; l < RB_LANES; ++l) q[l] = p[l] + p[l ^ o];
    memcpy(p, q, sizeof(p));
  }
  return p[0];
}

static void rb_unit(const float* x, float* u, int d) {
  const float den = fmaxf(sqrtf(rb_dot(x, x, d)), 1e-12f);
  for (int i = 0; i < d; ++i) u[i] = x[i] / den;
}

/* Squared norms (canonical dot) of bf16 rows. */
void orc_rb_norms(const uint16_t* x, int64_t rows, int d, float* out) {
  float v[RB_MAX_D];
  for (int64_t r = 0; r < rows; ++r) {
    for (int i = 0; i < d; ++i) v[i] = rb_bf16(x[r * d + i]);
    out[r] = rb_dot(v, v, d);
  }
}

typedef struct {
  float score;
  int32_t id;
  int32_t pos;
} RbKey;

/* (score, id) order; IEEE comparisons, so -0 and +0 tie and fall through to the id. */
static int rb_key_cmp(const void* a, const void* b) {
  const RbKey* x = (const RbKey*)a;
  const RbKey* y = (const RbKey*)b;
  if (x->score < y->score) return -1;
  if (x->score > y->score) return 1;
  return (x->id > y->id) - (x->id < y->id);
}

/* One internal node of the split topology: children [s0, s1) split at mid; tags >= 0 name the
 * internal child node, tags < 0 a finished child (-1 - child); slot indexes the landmark
 * weights the node receives from its parent. */
typedef struct {
  int s0, s1, mid, slot, ltag, rtag;
} RbTopo;

/* Breadth-first split topology of `children` children: returns the node count, children - 1.
 * For a power-of-two count the numbering is the heap's (node h has children 2h+1, 2h+2). */
static int rb_topology(int children, RbTopo* rec) {
  if (children < 2) return 0;
  int count = 1;
  rec[0].s0 = 0;
  rec[0].s1 = children;
  rec[0].slot = 0;
  for (int k = 0; k < count; ++k) {
    RbTopo* r = &rec[k];
    r->mid = r->s0 + (r->s1 - r->s0 + 1) / 2;
    const int a[2] = {r->s0, r->mid}, b[2] = {r->mid, r->s1};
    int tag[2];
    for (int side = 0; side < 2; ++side) {
      if (b[side] - a[side] == 1) {
        tag[side] = -1 - a[side];
      } else {
        rec[count].s0 = a[side];
        rec[count].s1 = b[side];
        rec[count].slot = 2 * k + 1 + side;
        tag[side] = count++;
      }
    }
    r->ltag = tag[0];
    r->rtag = tag[1];
  }
  return count;
}

/* Proxy controls (landmark_v2_terminal.py:43-50, 62-148): mean-update passes (0, 1, 2 or 4;
 * with 0 one assignment pass still hands the children their landmark weights and the seeds
 * give the direction) and the seed rule (farthest valid pair, or the lowest and highest
 * valid landmark).  Updates are the capacity-weighted means. */
typedef struct {
  int iterations, endpoint_seeds;
} RbProxy;

static const RbProxy rb_default_proxy = {2, 0};

/* Proxy tree over 32 landmark centers: directions [children-1][d] by topology node. */
static void rb_proxy_tree(const float* x, const int32_t* weights, const int64_t* caps, int children, int d,
                          const RbProxy* proxy, float* dirs) {
  static float n[RB_LANDMARKS][RB_MAX_D];
  static float dist[RB_LANDMARKS][RB_LANDMARKS];
  static int64_t act[2 * RB_MAX_CHILDREN][RB_LANDMARKS];
  RbTopo topo[RB_MAX_CHILDREN];
  const int nodes = rb_topology(children, topo);
  for (int i = 0; i < RB_LANDMARKS; ++i) rb_unit(x + (int64_t)i * d, n[i], d);
  for (int i = 0; i < RB_LANDMARKS; ++i)
    for (int k = i + 1; k < RB_LANDMARKS; ++k) dist[i][k] = 1.0f - rb_dot(n[i], n[k], d);
  for (int i = 0; i < RB_LANDMARKS; ++i) act[0][i] = weights[i];
  for (int h = 0; h < nodes; ++h) {
    const int slot = topo[h].slot, start = topo[h].s0, mid = topo[h].mid, end = topo[h].s1;
    {
      int64_t lc = 0, rc = 0;
      for (int c = start; c < mid; ++c) lc += caps[c];
      for (int c = mid; c < end; ++c) rc += caps[c];
      int nvalid = 0, only = -1;
      for (int i = 0; i < RB_LANDMARKS; ++i)
        if (act[slot][i] > 0) {
          ++nvalid;
          if (only < 0) only = i;
        }
      if (only < 0) only = 0;
      int first = only, second = only;
      if (nvalid >= 2 && proxy->endpoint_seeds) {
        for (int i = RB_LANDMARKS - 1; i >= 0; --i)
          if (act[slot][i] > 0) {
            second = i;
            break;
          }
      } else if (nvalid >= 2) {
        /* first maximum in row-major (i, k) order over valid pairs i < k */
        float best = -INFINITY;
        int found = 0;
        for (int i = 0; i < RB_LANDMARKS; ++i) {
          if (act[slot][i] <= 0) continue;
          for (int k = i + 1; k < RB_LANDMARKS; ++k) {
            if (act[slot][k] <= 0) continue;
            if (!found || dist[i][k] > best) {
              best = dist[i][k];
              first = i;
              second = k;
              found = 1;
            }
          }
        }
      }
      float left[RB_MAX_D], right[RB_MAX_D], ul[RB_MAX_D], ur[RB_MAX_D], dir[RB_MAX_D];
      memcpy(left, x + (int64_t)first * d, sizeof(float) * d);
      memcpy(right, x + (int64_t)second * d, sizeof(float) * d);
      int64_t lw[RB_LANDMARKS], rw[RB_LANDMARKS];
      const int rounds = proxy->iterations > 0 ? proxy->iterations : 1;
      for (int it = 0; it < rounds; ++it) {
        rb_unit(left, ul, d);
        rb_unit(right, ur, d);
        for (int i = 0; i < d; ++i) dir[i] = ur[i] - ul[i];
        RbKey key[RB_LANDMARKS];
        for (int i = 0; i < RB_LANDMARKS; ++i) {
          key[i].score = rb_dot(n[i], dir, d);
          key[i].id = i;
          key[i].pos = i;
        }
        qsort(key, RB_LANDMARKS, sizeof(RbKey), rb_key_cmp); /* ties by landmark index: a stable sort */
        int64_t before = 0;
        for (int r = 0; r < RB_LANDMARKS; ++r) {
          const int i = key[r].id;
          int64_t take = lc - before;
          if (take < 0) take = 0;
          if (take > act[slot][i]) take = act[slot][i];
          lw[i] = take;
          rw[i] = act[slot][i] - take;
          before += act[slot][i];
        }
        if (it >= proxy->iterations) break; /* zero updates: one assignment, seeds kept */
        for (int e = 0; e < d; ++e) {
          float a = 0.f, b = 0.f;
          for (int i = 0; i < RB_LANDMARKS; ++i) {
            a = fmaf((float)lw[i], x[(int64_t)i * d + e], a);
            b = fmaf((float)rw[i], x[(int64_t)i * d + e], b);
          }
          left[e] = a / (float)lc;
          right[e] = b / (float)rc;
        }
      }
      rb_unit(left, ul, d);
      rb_unit(right, ur, d);
      for (int i = 0; i < d; ++i) dirs[(int64_t)h * d + i] = ur[i] - ul[i];
      for (int i = 0; i < RB_LANDMARKS; ++i) {
        act[2 * h + 1][i] = lw[i];
        act[2 * h + 2][i] = rw[i];
      }
    }
  }
}

/* Split one node: ids[n] (node order) -> out[n] grouped by child, stable. */
static int rb_split_node(const uint16_t* x, int d, const int32_t* ids, int64_t n, const int64_t* caps, int children,
                         const RbProxy* proxy, int32_t* out) {
  float centers[RB_LANDMARKS * RB_MAX_D];
  int32_t weights[RB_LANDMARKS];
  for (int i = 0; i < RB_LANDMARKS; ++i) {
    const int64_t start = (int64_t)i * n / RB_LANDMARKS, end = (int64_t)(i + 1) * n / RB_LANDMARKS;
    const int64_t p = start + (end - start) / 2;
    weights[i] = (int32_t)(end - start);
    const uint16_t* row = x + (int64_t)ids[p] * d;
    for (int e = 0; e < d; ++e) centers[i * d + e] = rb_bf16(row[e]);
  }
  float* dirs = (float*)malloc(sizeof(float) * (size_t)(children - 1) * d);
  float* scores = (float*)malloc(sizeof(float) * (size_t)n * (children - 1));
  int16_t* node = (int16_t*)calloc((size_t)n, sizeof(int16_t)); /* topology node, or -1 - child */
  RbKey* keys = (RbKey*)malloc(sizeof(RbKey) * (size_t)n);
  if (!dirs || !scores || !node || !keys) {
    free(dirs), free(scores), free(node), free(keys);
    return -1;
  }
  rb_proxy_tree(centers, weights, caps, children, d, proxy, dirs);
  float v[RB_MAX_D], u[RB_MAX_D];
  for (int64_t t = 0; t < n; ++t) {
    const uint16_t* row = x + (int64_t)ids[t] * d;
    for (int e = 0; e < d; ++e) v[e] = rb_bf16(row[e]);
    rb_unit(v, u, d);
    for (int h = 0; h < children - 1; ++h) scores[t * (children - 1) + h] = rb_dot(u, dirs + (int64_t)h * d, d);
  }
  /* exact capacity routing, topology node by topology node (breadth first) */
  RbTopo topo[RB_MAX_CHILDREN];
  const int nodes = rb_topology(children, topo);
  for (int h = 0; h < nodes; ++h) {
    int64_t lc = 0;
    for (int c = topo[h].s0; c < topo[h].mid; ++c) lc += caps[c];
    int64_t m = 0;
    for (int64_t t = 0; t < n; ++t)
      if (node[t] == h) {
        keys[m].score = scores[t * (children - 1) + h];
        keys[m].id = ids[t];
        keys[m].pos = (int32_t)t;
        ++m;
      }
    qsort(keys, (size_t)m, sizeof(RbKey), rb_key_cmp);
    for (int64_t r = 0; r < m; ++r) node[keys[r].pos] = (int16_t)(r < lc ? topo[h].ltag : topo[h].rtag);
  }
  /* stable partition by label */
  int64_t offset = 0;
  for (int c = 0; c < children; ++c) {
    const int label = -1 - c;
    int64_t w = offset;
    for (int64_t t = 0; t < n; ++t)
      if (node[t] == label) out[w++] = ids[t];
    if (w - offset != caps[c]) {
      free(dirs), free(scores), free(node), free(keys);
      return -2;
    }
    offset += caps[c];
  }
  free(dirs), free(scores), free(node), free(keys);
  return 0;
}

/*
 * Full tree for `rows` independent rows of x [rows, tokens, d] bf16 (d a multiple of 32,
 * at most 256).  root_order [tokens]: the initial order (raster ids).  schedule: the
 * hierarchy, encoded as [levels, then per level: entries, then per entry: leaves, children,
 * budget_0 .. budget_{children-1}].  perm [rows, tokens] int32: leaves in order, then the
 * N mod 64 protected remainder tokens in root order.  Returns 0, or a negative error.
 */
int orc_rb_tree_proxy(const uint16_t* x, int rows, int tokens, int d, const int32_t* root_order,
                      const int32_t* schedule, int iterations, int endpoint_seeds, const int32_t* frozen,
                      int32_t* perm) {
  if (d % RB_LANES != 0 || d > RB_MAX_D || tokens < 64) return -10;
  if (iterations != 0 && iterations != 1 && iterations != 2 && iterations != 4) return -15;
  const RbProxy proxy_controls = {iterations, endpoint_seeds != 0};
  const RbProxy* proxy = &proxy_controls;
  const int rem = tokens % 64;
  const int64_t active = tokens - rem;
  int32_t* cur = (int32_t*)malloc(sizeof(int32_t) * (size_t)tokens);
  int32_t* nxt = (int32_t*)malloc(sizeof(int32_t) * (size_t)tokens);
  float* norms = (float*)malloc(sizeof(float) * (size_t)tokens);
  uint8_t* excluded = (uint8_t*)malloc((size_t)tokens);
  int64_t* seg_start = (int64_t*)malloc(sizeof(int64_t) * (size_t)(tokens / 64 + 1));
  int64_t* seg_leaves = (int64_t*)malloc(sizeof(int64_t) * (size_t)(tokens / 64 + 1));
  int64_t* nseg_start = (int64_t*)malloc(sizeof(int64_t) * (size_t)(tokens / 64 + 1));
  int64_t* nseg_leaves = (int64_t*)malloc(sizeof(int64_t) * (size_t)(tokens / 64 + 1));
  int rc = 0;
  if (!cur || !nxt || !norms || !excluded || !seg_start || !seg_leaves || !nseg_start || !nseg_leaves) {
    rc = -11;
    goto done;
  }
  for (int r = 0; r < rows && rc == 0; ++r) {
    const uint16_t* xr = x + (int64_t)r * tokens * d;
    int32_t* pr = perm + (int64_t)r * tokens;
    memset(excluded, 0, (size_t)tokens);
    if (rem && frozen) { /* the caller's protected remainder (landmark_tree_clustering.py:103-119) */
      for (int k = 0; k < rem; ++k) {
        const int32_t id = frozen[(int64_t)r * rem + k];
        if (id < 0 || id >= tokens || excluded[id]) {
          rc = -16;
          break;
        }
        excluded[id] = 1;
      }
      if (rc) break;
    } else if (rem) {
      orc_rb_norms(xr, tokens, d, norms);
      for (int k = 0; k < rem; ++k) {
        int best = -1;
        for (int t = 0; t < tokens; ++t)
          if (!excluded[t] && (best < 0 || norms[t] > norms[best])) best = t;
        excluded[best] = 1;
      }
    }
    int64_t a = 0, e = active;
    for (int i = 0; i < tokens; ++i) {
      const int32_t id = root_order[i];
      if (excluded[id])
        pr[e++] = id;
      else
        cur[a++] = id;
    }
    int nseg = 1;
    seg_start[0] = 0;
    seg_leaves[0] = active / 64;
    int pos = 1;
    const int levels = schedule[0];
    for (int level = 0; level < levels && rc == 0; ++level) {
      const int entries = schedule[pos];
      const int level_pos = pos + 1;
      int p = level_pos;
      for (int en = 0; en < entries; ++en) p += 2 + schedule[p + 1];
      pos = p;
      int nn = 0;
      memcpy(nxt, cur, sizeof(int32_t) * (size_t)active);
      for (int s = 0; s < nseg && rc == 0; ++s) {
        if (seg_leaves[s] <= 1) {
          nseg_start[nn] = seg_start[s];
          nseg_leaves[nn++] = seg_leaves[s];
          continue;
        }
        int q = level_pos, found = -1;
        for (int en = 0; en < entries; ++en) {
          if (schedule[q] == seg_leaves[s]) {
            found = q;
            break;
          }
          q += 2 + schedule[q + 1];
        }
        if (found < 0) {
          rc = -12;
          break;
        }
        const int children = schedule[found + 1];
        if (children < 2 || children > RB_MAX_CHILDREN) {
          rc = -13;
          break;
        }
        int64_t caps[RB_MAX_CHILDREN];
        int64_t off = seg_start[s];
        for (int c = 0; c < children; ++c) {
          caps[c] = 64 * (int64_t)schedule[found + 2 + c];
          nseg_start[nn] = off;
          nseg_leaves[nn++] = schedule[found + 2 + c];
          off += caps[c];
        }
        rc = rb_split_node(xr, d, cur + seg_start[s], 64 * seg_leaves[s], caps, children, proxy, nxt + seg_start[s]);
      }
      int32_t* t = cur;
      cur = nxt;
      nxt = t;
      nseg = nn;
      memcpy(seg_start, nseg_start, sizeof(int64_t) * (size_t)nn);
      memcpy(seg_leaves, nseg_leaves, sizeof(int64_t) * (size_t)nn);
    }
    for (int s = 0; s < nseg && rc == 0; ++s)
      if (seg_leaves[s] > 1) rc = -14; /* schedule ended before every node became a leaf */
    memcpy(pr, cur, sizeof(int32_t) * (size_t)active);
  }
done:
  free(cur), free(nxt), free(norms), free(excluded);
  free(seg_start), free(seg_leaves), free(nseg_start), free(nseg_leaves);
  return rc;
}

/* The production proxy controls: two mean updates from the farthest pair. */
int orc_rb_tree(const uint16_t* x, int rows, int tokens, int d, const int32_t* root_order, const int32_t* schedule,
                int32_t* perm) {
  return orc_rb_tree_proxy(x, rows, tokens, d, root_order, schedule, rb_default_proxy.iterations,
                           rb_default_proxy.endpoint_seeds, NULL, perm);
}
