"""CPU tests of the streaming synthetic-data tooling (coraanns_b200.synthetic) used by the
large-configuration bench runs and full-size GPU tests: the two-pass streaming build equals
the in-memory builder on the same vectors, and the streamed ground truth and exact scores
equal brute force."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import py_oracle as po


@pytest.mark.parametrize("metric,zipf", [(0, None), (1, 1.1)])
def test_stream_build_equals_in_memory_build(metric, zipf):
    from coraanns_b200 import builder, synthetic
    mix = synthetic.Mixture(5000, 96, 16, 0.3, seed=11, normalise=metric == 1, zipf_s=zipf,
                            device="cpu", chunk=1024)
    cent = synthetic.train_centroids(mix, 16, sample=3000)
    sd = synthetic.build_index_stream(mix, cent, metric=metric, seed=5)
    x = torch.cat([mix.chunk_at(j)[0] for j in range(mix.n_chunks)])
    lab = synthetic._nearest(x, cent, (cent * cent).sum(1))
    ref = builder.build_index(x, cent, lab, seed=5, metric=metric)
    for key in ("short_data", "short_factors", "long_codes", "ex_factors", "ids", "sizes",
                "centroids", "rotator"):
        assert np.array_equal(np.asarray(sd[key]), np.asarray(ref[key])), key
    assert sd["metric"] == metric
    if zipf:  # heavy-tailed component weights: the largest cluster dominates
        assert sd["sizes"].max() > 4 * np.median(sd["sizes"])


@pytest.mark.parametrize("metric", [0, 1])
def test_stream_ground_truth_and_scores(metric):
    from coraanns_b200 import synthetic
    mix = synthetic.Mixture(3000, 32, 8, 0.3, seed=3, normalise=metric == 1, device="cpu",
                            chunk=700)
    q = mix.queries(20, 0.05)
    ids, d = synthetic.ground_truth_stream(mix, q, 10, metric=metric, keep=16)
    x = torch.cat([mix.chunk_at(j)[0] for j in range(mix.n_chunks)])
    want_i, want_d = po.exact_knn(x.numpy(), q.numpy(), 10, metric)
    assert np.array_equal(ids.numpy(), want_i.astype(np.int64))
    assert np.allclose(d.numpy(), want_d, rtol=1e-12, atol=1e-12)
    sc = synthetic.exact_scores(mix, q, ids, metric)
    assert np.allclose(sc.numpy(), want_d, rtol=1e-12, atol=1e-12)
    assert synthetic.distance_recall(ids, d, ids.numpy(), sc, 10) == 1.0


def _component_fixture(world=3):
    from coraanns_b200 import synthetic
    from coraanns_b200.shard import shard_plan
    mix = synthetic.ComponentShards(30_000, 40, 64, 0.25, seed=11, device="cpu")
    owner = shard_plan(mix.counts, world)
    return mix, owner


def test_shard_build_equals_slice_of_whole_build():
    """Each shard built alone from its own clusters (per-shard generation) holds exactly the
    arrays the whole index's build gives that shard (shard_search_data)."""
    from coraanns_b200 import builder, synthetic
    from coraanns_b200.shard import shard_search_data
    mix, owner = _component_fixture()
    x, lab, gid = mix.clusters(np.arange(mix.ncomp))
    assert torch.equal(gid, torch.arange(mix.n))  # cluster-major ids
    # batches of whole clusters regenerate the same vectors
    xb = torch.cat([b[0] for b in mix.batches(rows=1000)])
    assert torch.equal(xb, x)
    full = builder.build_index(x, mix.centres, lab, seed=5)
    assert np.array_equal(full["sizes"].astype(np.int64), mix.counts)
    for r in range(3):
        want = shard_search_data(full, owner, r)
        got = synthetic.build_shard(mix, owner, r, seed=5)
        assert got["num"] == want["num"] > 0
        for key in ("centroids", "rotator", "short_data", "short_factors", "long_codes",
                    "ex_factors", "ids", "sizes"):
            assert np.asarray(got[key]).tobytes() == np.asarray(want[key]).tobytes(), key


def test_shard_ground_truth_merges_to_whole():
    from coraanns_b200 import synthetic
    mix, owner = _component_fixture()
    q = mix.queries(40, 0.05)
    parts = [synthetic.ground_truth_shard(mix, owner, r, q, 10) for r in range(3)]
    ids, d = synthetic.merge_topk(torch.cat([p[0] for p in parts], 1),
                                  torch.cat([p[1] for p in parts], 1), 10)
    best_d, best_i = synthetic._gt_init(q, 10)
    for x, _, gid in mix.batches(rows=5000):
        synthetic._gt_update(best_d, best_i, x, gid, q, 10, 0, 64, 2048)
    assert torch.equal(ids, best_i) and torch.equal(d, best_d)
    # exact scores of every returned id, each from its own shard
    sc = torch.stack([synthetic.exact_scores_shard(mix, owner, r, q, ids) for r in range(3)])
    assert torch.equal(sc.min(0).values, best_d)
