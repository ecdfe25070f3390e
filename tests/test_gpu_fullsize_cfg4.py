"""Full-size checks at BASELINE config 4: 88M x d768 unit vectors, inner product, nlist
32768, 10K queries, topk 100, vanguard 5, nprobe 32.

The base is a seeded unit-normalised Gaussian mixture generated chunk by chunk on the GPU
(coraanns_b200.synthetic; the 270 GB fp32 base never exists at once) and indexed by the
streamed builder. The whole 10K-query batch is checked through size-independent properties
(finite, ascending (distance, id) rows, unique ids, captured thresholds equal to the k-th
distance, a second search returning the same bytes), for both of the reference's scan
estimators; a seeded sample of queries is checked bit for bit against the C oracle on the
same in-memory index (ids, distances and candidate counts).
"""
from __future__ import annotations

import numpy as np
import pytest

import py_oracle as po

pytestmark = pytest.mark.gpu

N, DIM, NLIST, NQ, K, NPROBE, VANGUARD = 88_000_000, 768, 32768, 10_000, 100, 32, 5
SIGMA, QNOISE, SEED = 0.2, 0.05, 20261204


@pytest.fixture(scope="module")
def cfg4():
    import torch
    from coraanns_b200 import synthetic
    if torch.cuda.get_device_properties(0).total_memory < 150 * 2**30:
        pytest.skip("needs a GPU with the memory of a B200")
    dev = torch.device("cuda", 0)
    mix = synthetic.Mixture(N, DIM, NLIST, SIGMA, SEED, normalise=True, device=dev)
    cent = synthetic.train_centroids(mix, NLIST, sample=64 * NLIST)
    sd = synthetic.build_index_stream(mix, cent, metric=1, seed=SEED)
    q = mix.queries(NQ, QNOISE).cpu().numpy()
    del mix, cent
    torch.cuda.empty_cache()
    yield sd, q
    sd.clear()


@pytest.fixture(scope="module")
def engine(cfg4):
    import coraanns_b200 as cb
    sd, q = cfg4
    e = cb.HybridIndex(0)
    e.load_search_data(sd)
    e.set_vanguard_size(VANGUARD)
    e.prepare_workspace(NQ, K, NPROBE)
    e.reset_buffer(q)
    yield e
    e.close()


def _batch_properties(e, q):
    d, i = e.search(q, K, NPROBE)
    assert np.isfinite(d).all()                      # >= k candidates for every query
    dd = d[:, 1:] - d[:, :-1]                        # ascending (distance, id)
    assert ((dd > 0) | ((dd == 0) & (i[:, 1:] > i[:, :-1]))).all()
    srt = np.sort(i, axis=1)
    assert (srt[:, 1:] != srt[:, :-1]).all()         # unique ids
    assert (i < N).all()
    t = e.capture_thresholds(NQ)
    assert t.tobytes() == d[:, K - 1].copy().tobytes()
    d2, i2 = e.search(q, K, NPROBE)
    assert d2.tobytes() == d.tobytes() and np.array_equal(i2, i)
    return d, i, e.debug("cand_count", NQ)


@pytest.mark.parametrize("estimator", ["bitwise", "lut"])
def test_cfg4_batch_properties_and_oracle_sample(cfg4, engine, estimator):
    import coraanns_b200 as cb
    sd, q = cfg4
    assert engine.get_metric() == 1
    engine.set_ip_kernel_type(cb.KernelType.Bitwise if estimator == "bitwise"
                              else cb.KernelType.Lut4Bit)
    try:
        d, i, cand = _batch_properties(engine, q)
    finally:
        engine.set_ip_kernel_type(cb.KernelType.Bitwise)
    rng = np.random.default_rng(41)
    sample = np.sort(rng.choice(NQ, 24, replace=False))
    ref = po.OracleIndex(sd, lut=estimator == "lut").search(
        q[sample], K, NPROBE, vanguard=VANGUARD, with_details=True)
    assert np.array_equal(i[sample], ref["ids"])
    assert d[sample].tobytes() == ref["dist"].tobytes()
    assert np.array_equal(cand[sample].astype(np.uint64), ref["cand_count"])
