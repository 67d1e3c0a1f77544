// Near-duplicate graph over SSCD copy-detection edges: host C++17 behind a handle-based C ABI.
//
// Design: the edge list is validated once and turned into a CSR adjacency by a counting sort
// (two passes: degrees, then placement in edge order). Connected components come from a
// breadth-first sweep over that CSR, started at every still-unlabelled vertex in increasing id
// order, so each component's label is its smallest vertex id without any extra pass. Everything
// else (sizes, statistics, representative selection) reads the CSR; the caller copies results
// out through small accessors and frees the graph with sscd_graph_free.
//
// Edge records are the corpus file format {uint32 a; uint32 b; float32 score} (12 bytes, a < b,
// score >= threshold).
//
// Representatives: vertices are visited in a caller-given priority order. A visited vertex that
// is eligible, not protected and not yet assigned becomes a representative and takes every
// neighbour that is eligible, not protected and still unassigned (one hop only, so membership is
// never transitive). Protected eligible vertices represent themselves from the start and never
// take or join another group. Ineligible vertices get no representative.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <limits>
#include <new>
#include <vector>

namespace {

struct EdgeRecord {
  uint32_t a, b;
  float score;
};
static_assert(sizeof(EdgeRecord) == 12, "edge records are 12 bytes");

constexpr uint32_t kUnset = std::numeric_limits<uint32_t>::max();

thread_local char g_error[200] = "";

int fail(int code, const char* what, unsigned long long where = 0) {
  std::snprintf(g_error, sizeof(g_error), "%s (at %llu)", what, where);
  return code;
}

struct Graph {
  uint32_t n = 0;
  float threshold = 0.f;
  std::vector<uint64_t> row;          // CSR offsets [n + 1]
  std::vector<uint32_t> col;          // neighbours [2 m]
  std::vector<float> weight;          // scores [2 m]
  std::vector<uint32_t> label;        // smallest vertex id of the component
  std::vector<uint32_t> comp_size;    // size of the vertex's component
};

}  // namespace

extern "C" {

enum SscdStatus {
  SSCD_OK = 0,
  SSCD_TOO_MANY_VERTICES = -1,
  SSCD_BAD_EDGE = -2,        // endpoint out of range or not a < b
  SSCD_WEAK_EDGE = -3,       // score not finite or below the threshold
  SSCD_BAD_ORDER = -4,       // priority order names a vertex outside [0, n)
  SSCD_NO_MEMORY = -5,
  SSCD_NULL = -6,
};

struct SscdStats {
  uint64_t components, nontrivial_components, largest_component, vertices_with_edges, isolated_vertices,
      max_degree;
  uint64_t size_histogram[32];  // bin b: components whose size s has floor(log2 s) == b
};

struct SscdSelection {
  uint64_t eligible, representatives, suppressed, ineligible, protected_vertices;
};

const char* sscd_last_error(void) { return g_error; }

// Builds the graph; on success *out owns it (free with sscd_graph_free).
int sscd_graph_build(uint64_t n, const EdgeRecord* edges, uint64_t m, float threshold, void** out) {
  if (!out || (m && !edges)) return fail(SSCD_NULL, "null argument");
  *out = nullptr;
  if (n >= kUnset) return fail(SSCD_TOO_MANY_VERTICES, "vertex ids must fit in 32 bits", n);
  Graph* g = new (std::nothrow) Graph;
  if (!g) return fail(SSCD_NO_MEMORY, "out of memory");
  try {
    g->n = static_cast<uint32_t>(n);
    g->threshold = threshold;
    g->row.assign(n + 1, 0);
    for (uint64_t i = 0; i < m; ++i) {     // validate and count degrees (row[v + 1])
      const EdgeRecord& e = edges[i];
      if (e.a >= n || e.b >= n || e.a >= e.b) {
        delete g;
        return fail(SSCD_BAD_EDGE, "malformed edge", i);
      }
      if (!std::isfinite(e.score) || e.score < threshold) {
        delete g;
        return fail(SSCD_WEAK_EDGE, "edge score below threshold or not finite", i);
      }
      ++g->row[e.a + 1];
      ++g->row[e.b + 1];
    }
    for (uint64_t v = 0; v < n; ++v) g->row[v + 1] += g->row[v];
    g->col.resize(2 * m);
    g->weight.resize(2 * m);
    std::vector<uint64_t> next(g->row.begin(), g->row.end() - 1);
    for (uint64_t i = 0; i < m; ++i) {     // placement keeps edge order inside every row
      const EdgeRecord& e = edges[i];
      uint64_t p = next[e.a]++;
      g->col[p] = e.b;
      g->weight[p] = e.score;
      p = next[e.b]++;
      g->col[p] = e.a;
      g->weight[p] = e.score;
    }
    g->label.assign(n, kUnset);
    g->comp_size.assign(n, 0);
    std::vector<uint32_t> queue;
    queue.reserve(64);
    for (uint32_t s = 0; s < n; ++s) {     // BFS from each unlabelled vertex, ids ascending
      if (g->label[s] != kUnset) continue;
      queue.clear();
      queue.push_back(s);
      g->label[s] = s;
      for (size_t head = 0; head < queue.size(); ++head) {
        const uint32_t v = queue[head];
        for (uint64_t p = g->row[v]; p < g->row[v + 1]; ++p) {
          const uint32_t u = g->col[p];
          if (g->label[u] == kUnset) {
            g->label[u] = s;
            queue.push_back(u);
          }
        }
      }
      for (uint32_t v : queue) g->comp_size[v] = static_cast<uint32_t>(queue.size());
    }
  } catch (const std::bad_alloc&) {
    delete g;
    return fail(SSCD_NO_MEMORY, "out of memory");
  }
  *out = g;
  return SSCD_OK;
}

void sscd_graph_free(void* graph) { delete static_cast<Graph*>(graph); }

uint64_t sscd_graph_edges(const void* graph) { return static_cast<const Graph*>(graph)->col.size() / 2; }

// label[n], component_size[n] (either may be null).
int sscd_graph_components(const void* graph, uint32_t* label, uint32_t* component_size) {
  const Graph* g = static_cast<const Graph*>(graph);
  if (!g) return fail(SSCD_NULL, "null graph");
  if (label) std::memcpy(label, g->label.data(), sizeof(uint32_t) * g->n);
  if (component_size) std::memcpy(component_size, g->comp_size.data(), sizeof(uint32_t) * g->n);
  return SSCD_OK;
}

// offsets[n + 1], neighbors[2 m], scores[2 m].
int sscd_graph_adjacency(const void* graph, uint64_t* offsets, uint32_t* neighbors, float* scores) {
  const Graph* g = static_cast<const Graph*>(graph);
  if (!g || !offsets || (!g->col.empty() && (!neighbors || !scores))) return fail(SSCD_NULL, "null argument");
  std::memcpy(offsets, g->row.data(), sizeof(uint64_t) * (g->n + 1ull));
  std::memcpy(neighbors, g->col.data(), sizeof(uint32_t) * g->col.size());
  std::memcpy(scores, g->weight.data(), sizeof(float) * g->weight.size());
  return SSCD_OK;
}

int sscd_graph_stats(const void* graph, SscdStats* stats) {
  const Graph* g = static_cast<const Graph*>(graph);
  if (!g || !stats) return fail(SSCD_NULL, "null argument");
  std::memset(stats, 0, sizeof(SscdStats));
  for (uint32_t v = 0; v < g->n; ++v) {
    const uint64_t degree = g->row[v + 1] - g->row[v];
    (degree ? stats->vertices_with_edges : stats->isolated_vertices) += 1;
    stats->max_degree = std::max(stats->max_degree, degree);
    if (g->label[v] != v) continue;        // one visit per component: at its smallest vertex
    const uint32_t size = g->comp_size[v];
    stats->components += 1;
    stats->nontrivial_components += size > 1;
    stats->largest_component = std::max<uint64_t>(stats->largest_component, size);
    int bin = 31 - __builtin_clz(size);
    stats->size_histogram[bin] += 1;
  }
  return SSCD_OK;
}

// order[n] (priority; eligible vertices it does not list end up as their own representatives),
// eligible[n] / protect[n] (0/1, may be null: all eligible / none protected). Outputs representative[n] (kUnset for ineligible), direct_score[n] (score of the
// edge to the representative, 1 for representatives, NaN for ineligible), group_size[n]
// (members of each representative's group, 0 elsewhere).
int sscd_graph_select(const void* graph, const uint32_t* order, const uint8_t* eligible, const uint8_t* protect,
                      uint32_t* representative, float* direct_score, uint32_t* group_size, SscdSelection* summary) {
  const Graph* g = static_cast<const Graph*>(graph);
  if (!g || !order || !representative || !direct_score || !group_size || !summary)
    return fail(SSCD_NULL, "null argument");
  const uint32_t n = g->n;
  auto ok = [&](uint32_t v) { return !eligible || eligible[v]; };
  auto fixed = [&](uint32_t v) { return protect && protect[v]; };
  std::fill(representative, representative + n, kUnset);
  std::fill(direct_score, direct_score + n, std::numeric_limits<float>::quiet_NaN());
  std::fill(group_size, group_size + n, 0u);
  std::memset(summary, 0, sizeof(SscdSelection));
  for (uint32_t v = 0; v < n; ++v)
    if (ok(v) && fixed(v)) {
      representative[v] = v;
      direct_score[v] = 1.f;
    }
  for (uint64_t k = 0; k < n; ++k) {
    const uint32_t v = order[k];
    if (v >= n) return fail(SSCD_BAD_ORDER, "priority order holds an out-of-range vertex", k);
    if (!ok(v) || fixed(v) || representative[v] != kUnset) continue;
    representative[v] = v;
    direct_score[v] = 1.f;
    for (uint64_t p = g->row[v]; p < g->row[v + 1]; ++p) {
      const uint32_t u = g->col[p];
      if (!ok(u) || fixed(u)) continue;
      if (representative[u] == kUnset) {
        representative[u] = v;
        direct_score[u] = g->weight[p];
      } else if (representative[u] == v && u != v) {
        direct_score[u] = std::max(direct_score[u], g->weight[p]);   // parallel edges keep the best
      }
    }
  }
  for (uint32_t v = 0; v < n; ++v) {
    if (!ok(v)) {
      summary->ineligible += 1;
      continue;
    }
    if (representative[v] == kUnset) {   // eligible but missing from the order: its own group
      representative[v] = v;
      direct_score[v] = 1.f;
    }
    const uint32_t r = representative[v];
    group_size[r] += 1;
    summary->eligible += 1;
    (r == v ? summary->representatives : summary->suppressed) += 1;
    summary->protected_vertices += fixed(v);
  }
  return SSCD_OK;
}

}  // extern "C"
