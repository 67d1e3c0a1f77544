// Near-duplicate graph arithmetic for SSCD copy-detection edges (host C++, C ABI).
//
// Input edges use the corpus file record {uint32 a; uint32 b; float32 score} (12 bytes, a < b,
// score >= threshold). The library provides:
//   * connected components with a disjoint-set forest (path halving, union by size);
//   * per-vertex component label (= smallest vertex id of the component), component size,
//     degree, a summary and a log2 histogram of component sizes;
//   * a CSR adjacency (offsets from the degrees, neighbours + scores filled in edge order);
//   * greedy representative selection: vertices are visited in a caller-given priority order;
//     an unassigned eligible vertex becomes a representative and claims its unassigned eligible
//     neighbours (one hop, no transitive chains); protected vertices always represent
//     themselves and neither claim nor get claimed.
// Every entry point validates its inputs and returns 0 on success or a distinct error code.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>

namespace {

struct Edge {
  uint32_t a, b;
  float score;
};
static_assert(sizeof(Edge) == 12, "edge records are 12 bytes");

constexpr uint32_t kNone = std::numeric_limits<uint32_t>::max();

uint32_t root_of(uint32_t v, uint32_t* parent) {
  while (parent[v] != v) {
    parent[v] = parent[parent[v]];  // path halving
    v = parent[v];
  }
  return v;
}

bool valid_edge(const Edge& e, uint64_t n) { return e.a < n && e.b < n && e.a < e.b; }

}  // namespace

extern "C" {

// parent[i] = i, size[i] = 1, degree[i] = 0. Error 1: n does not fit 32-bit vertex ids.
int sscd_init(uint64_t n, uint32_t* parent, uint32_t* size, uint64_t* degree) {
  if (n >= kNone) return 1;
  for (uint64_t i = 0; i < n; ++i) {
    parent[i] = static_cast<uint32_t>(i);
    size[i] = 1;
    degree[i] = 0;
  }
  return 0;
}

// Union the endpoints of m edges and count degrees. Error 2: malformed edge or score below
// the threshold (or not finite).
int sscd_union(uint64_t n, uint64_t m, const Edge* edges, uint32_t* parent, uint32_t* size, uint64_t* degree,
               float threshold) {
  for (uint64_t i = 0; i < m; ++i) {
    const Edge& e = edges[i];
    if (!valid_edge(e, n) || !std::isfinite(e.score) || e.score < threshold) return 2;
    degree[e.a] += 1;
    degree[e.b] += 1;
    uint32_t ra = root_of(e.a, parent), rb = root_of(e.b, parent);
    if (ra == rb) continue;
    if (size[ra] < size[rb]) std::swap(ra, rb);
    parent[rb] = ra;
    size[ra] += size[rb];
  }
  return 0;
}

// Labels, sizes, CSR offsets[n + 1], summary[6] = {components, non-singleton components,
// largest component, vertices with edges, isolated vertices, max degree} and histogram[32]
// (bin b counts components with floor(log2(size)) == b).
int sscd_components(uint64_t n, uint32_t* parent, const uint32_t* size, const uint64_t* degree, uint32_t* label,
                    uint32_t* component_size, uint64_t* offsets, uint64_t* summary, uint64_t* histogram) {
  std::fill(summary, summary + 6, uint64_t(0));
  std::fill(histogram, histogram + 32, uint64_t(0));
  std::fill(label, label + n, kNone);
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t r = root_of(static_cast<uint32_t>(i), parent);
    parent[i] = r;                                  // flatten
    label[r] = std::min(label[r], static_cast<uint32_t>(i));
  }
  offsets[0] = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t r = parent[i];
    label[i] = label[r];
    component_size[i] = size[r];
    offsets[i + 1] = offsets[i] + degree[i];
    summary[degree[i] ? 3 : 4] += 1;
    summary[5] = std::max(summary[5], degree[i]);
    if (r == i) {
      summary[0] += 1;
      if (size[i] > 1) summary[1] += 1;
      summary[2] = std::max<uint64_t>(summary[2], size[i]);
      int bin = 0;
      for (uint32_t s = size[i]; s > 1; s >>= 1) ++bin;
      histogram[bin] += 1;
    }
  }
  return 0;
}

// Fill neighbours/scores of the CSR rows (cursor[i] starts at offsets[i]).
// Error 3: malformed edge; error 4: a row overflows its degree.
int sscd_fill(uint64_t n, uint64_t m, const Edge* edges, const uint64_t* offsets, uint64_t* cursor,
              uint32_t* neighbors, float* scores) {
  for (uint64_t i = 0; i < m; ++i) {
    const Edge& e = edges[i];
    if (!valid_edge(e, n)) return 3;
    const uint64_t ia = cursor[e.a]++, ib = cursor[e.b]++;
    if (ia >= offsets[e.a + 1] || ib >= offsets[e.b + 1]) return 4;
    neighbors[ia] = e.b;
    scores[ia] = e.score;
    neighbors[ib] = e.a;
    scores[ib] = e.score;
  }
  return 0;
}

// Greedy one-hop representatives (see the header). representative[i] = kNone for ineligible
// vertices; direct_score[i] = best score to its representative (1 for representatives);
// group_size[r] = members of r's group; summary[5] = {eligible, representatives, suppressed,
// ineligible, protected}. Error 5: order holds an out-of-range vertex; 6: bad neighbour or
// score; 7: inconsistent result.
int sscd_representatives(uint64_t n, const uint64_t* offsets, const uint32_t* neighbors, const float* scores,
                         const uint32_t* order, const uint8_t* eligible, const uint8_t* protect,
                         uint32_t* representative, float* direct_score, uint32_t* group_size, uint64_t* summary,
                         float threshold) {
  std::fill(representative, representative + n, kNone);
  std::fill(direct_score, direct_score + n, std::numeric_limits<float>::quiet_NaN());
  std::fill(group_size, group_size + n, 0u);
  std::fill(summary, summary + 5, uint64_t(0));
  for (uint64_t i = 0; i < n; ++i) {
    if (eligible[i] && protect[i]) {
      representative[i] = static_cast<uint32_t>(i);
      direct_score[i] = 1.f;
    }
  }
  for (uint64_t k = 0; k < n; ++k) {
    const uint32_t v = order[k];
    if (v >= n) return 5;
    if (!eligible[v] || protect[v] || representative[v] != kNone) continue;
    representative[v] = v;
    direct_score[v] = 1.f;
    for (uint64_t j = offsets[v]; j < offsets[v + 1]; ++j) {
      const uint32_t u = neighbors[j];
      const float s = scores[j];
      if (u >= n || !std::isfinite(s) || s < threshold) return 6;
      if (!eligible[u] || protect[u]) continue;
      if (representative[u] == kNone) {
        representative[u] = v;
        direct_score[u] = s;
      } else if (representative[u] == v) {
        direct_score[u] = std::max(direct_score[u], s);
      }
    }
  }
  for (uint64_t i = 0; i < n; ++i) {
    if (!eligible[i]) {
      summary[3] += 1;
      continue;
    }
    const uint32_t r = representative[i];
    if (r >= n || representative[r] != r || !eligible[r]) return 7;
    group_size[r] += 1;
    summary[0] += 1;
    summary[r == i ? 1 : 2] += 1;
    if (protect[i]) summary[4] += 1;
  }
  return 0;
}

}  // extern "C"
