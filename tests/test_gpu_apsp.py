"""APSP by repeated squaring: distances against Floyd-Warshall on the CPU,
each squaring bit-exact against the oracle, and reconstructed paths valid."""
import numpy as np
import pytest
import torch

from oracle import tg_oracle as O
from tropical_gemm.apsp import all_pairs_shortest_paths, reconstruct_path, I32_INF, squarings_needed

pytestmark = pytest.mark.gpu


def _graph(n, density, seed):
    rng = np.random.default_rng(seed)
    mask = rng.random((n, n)) < density
    w = rng.integers(1, 1001, (n, n)).astype(np.int32)
    d = np.where(mask, w, I32_INF).astype(np.int32)
    np.fill_diagonal(d, 0)
    return d


def _floyd(d):
    x = d.astype(np.int64).copy()
    x[x >= I32_INF] = 1 << 40
    for k in range(x.shape[0]):
        x = np.minimum(x, x[:, k:k + 1] + x[k:k + 1, :])
    x[x >= I32_INF] = I32_INF
    return x.astype(np.int32)


@pytest.mark.parametrize("n,density", [(5, 0.5), (64, 0.05), (300, 0.02)])
def test_apsp_matches_floyd_and_oracle(n, density):
    d = _graph(n, density, n)
    dist, ams = all_pairs_shortest_paths(torch.from_numpy(d).cuda())
    assert len(ams) == squarings_needed(n)
    cur = d
    for t, am in enumerate(ams):   # every squaring is the reference's GEMM, bit for bit
        nxt, am0 = O.gemm("minplus", cur, cur)
        assert np.array_equal(am.cpu().numpy(), am0)
        cur = nxt
    assert np.array_equal(dist.cpu().numpy(), cur)
    assert np.array_equal(dist.cpu().numpy(), _floyd(d))
    rng = np.random.default_rng(1)
    for _ in range(20):
        i, j = rng.integers(0, n, 2)
        if dist[i, j] >= I32_INF or i == j:
            continue
        path = reconstruct_path(int(i), int(j), ams)
        assert path[0] == i and path[-1] == j
        assert sum(int(d[a, b]) for a, b in zip(path, path[1:])) == int(dist[i, j])


def test_reference_example_graph_f64():
    """The 5-node graph of crates/tropical-gemm/examples/shortest_path.rs."""
    inf = np.inf
    d = np.array([[0, 3, inf, 7, inf], [inf, 0, 2, inf, inf], [inf, inf, 0, 1, 5],
                  [inf, inf, inf, 0, 2], [inf, inf, inf, inf, 0]], dtype=np.float64)
    dist, ams = all_pairs_shortest_paths(torch.from_numpy(d).cuda(), squarings=2)
    dist = dist.cpu().numpy()
    assert dist[0, 4] == 8 and dist[0, 2] == 5 and dist[1, 4] == 5
    assert reconstruct_path(0, 2, ams) == [0, 1, 2]
