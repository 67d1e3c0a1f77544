"""SSCD native graph library and exact pair search (CPU, with a GPU variant of the search)."""

import numpy as np
import pytest

from cq_pretrain_b200.corpus.sscd import EDGE_DTYPE, Graph, exact_pairs


def _edges(pairs):
    e = np.zeros(len(pairs), EDGE_DTYPE)
    for k, (a, b, s) in enumerate(pairs):
        e[k] = (a, b, s)
    return e


def test_components_csr_and_representatives():
    edges = _edges([(0, 1, 0.9), (1, 2, 0.8), (4, 5, 0.95), (0, 2, 0.85)])
    g = Graph(7, edges, 0.7)
    assert g.label.tolist() == [0, 0, 0, 3, 4, 4, 6]
    assert g.component_size.tolist() == [3, 3, 3, 1, 2, 2, 1]
    assert g.summary == dict(components=4, nontrivial_components=2, largest_component=3, vertices_with_edges=5,
                             isolated_vertices=2, max_degree=2)
    assert g.histogram[0] == 2 and g.histogram[1] == 2   # sizes 1,1 -> bin 0; 2,3 -> bin 1
    assert g.offsets.tolist() == [0, 2, 4, 6, 6, 7, 8, 8]
    assert sorted(g.neighbors[0:2].tolist()) == [1, 2]
    # priority: vertex 1 first claims 0 and 2 (one hop); 5 before 4
    rep, direct, group, summary = g.representatives(order=[1, 5, 0, 2, 3, 4, 6])
    assert rep.tolist() == [1, 1, 1, 3, 5, 5, 6]
    assert np.isclose(direct[0], 0.9) and np.isclose(direct[2], 0.8) and direct[1] == 1.0
    assert group[1] == 3 and summary["suppressed"] == 3 and summary["representatives"] == 4
    # protected vertices keep themselves and are never claimed; ineligible ones are skipped
    rep, _, _, summary = g.representatives(order=[1, 5, 0, 2, 3, 4, 6], protect=[0, 0, 1, 0, 0, 0, 0],
                                           eligible=[1, 1, 1, 1, 1, 1, 0])
    assert rep[2] == 2 and rep[0] == 1 and rep[6] == np.iinfo(np.uint32).max and summary["protected"] == 1


def test_graph_rejects_bad_edges():
    with pytest.raises(ValueError, match="below threshold"):
        Graph(3, _edges([(0, 1, 0.5)]), 0.7)
    with pytest.raises(ValueError):
        Graph(3, _edges([(2, 1, 0.9)]), 0.7)


def test_exact_pairs_cpu_matches_bruteforce():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((300, 32)).astype(np.float32)
    x[150:160] = x[0] + 0.05 * rng.standard_normal((10, 32))   # a cluster of near duplicates
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    edges = exact_pairs(x, x, 0.9, tile=128, device="cpu")
    sims = x @ x.T
    want = {(i, j) for i in range(300) for j in range(i + 1, 300) if sims[i, j] >= 0.9}
    assert {(int(a), int(b)) for a, b in zip(edges["a"], edges["b"])} == want and len(want) >= 45
    g = Graph(300, edges, 0.9)
    assert g.summary["largest_component"] == 11


@pytest.mark.gpu
def test_exact_pairs_gpu_matches_cpu():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1024, 64)).astype(np.float32)
    x[512:540] = x[3] + 0.03 * rng.standard_normal((28, 64))
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    gpu = exact_pairs(x, x, 0.85, tile=256, device="cuda")
    cpu = exact_pairs(x, x, 0.85, tile=256, device="cpu")
    assert set(zip(gpu["a"].tolist(), gpu["b"].tolist())) == set(zip(cpu["a"].tolist(), cpu["b"].tolist()))
