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
