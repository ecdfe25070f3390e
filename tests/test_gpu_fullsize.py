"""Full-size checks at BASELINE config 2 (10M x d96, nlist 4096, 10K queries, nprobe 8).

The whole 10K-query batch is checked through size-independent properties (sorted (distance,
id) rows, unique ids, captured thresholds equal to the k-th distance, a second search and a
2-shard search returning the same bytes); a seeded sample of queries is checked bit for bit
against the C oracle on the same index.
"""
from __future__ import annotations

import numpy as np
import pytest

import py_oracle as po

pytestmark = pytest.mark.gpu

N, DIM, NLIST, NQ, K, NPROBE = 10_000_000, 96, 4096, 10_000, 10, 8


@pytest.fixture(scope="module")
def fullsize():
    import torch
    from coraanns_b200 import builder
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(20261207)
    centres = torch.randn(NLIST, DIM, generator=g, device=dev)
    base = torch.empty(N, DIM, device=dev)
    lab = torch.empty(N, dtype=torch.int64, device=dev)
    for s in range(0, N, 1 << 21):
        e = min(N, s + (1 << 21))
        lab[s:e] = torch.randint(0, NLIST, (e - s,), generator=g, device=dev)
        base[s:e] = centres[lab[s:e]] + 0.25 * torch.randn(e - s, DIM, generator=g, device=dev)
    qlab = torch.randint(0, NLIST, (NQ,), generator=g, device=dev)
    q = centres[qlab] + 0.25 * torch.randn(NQ, DIM, generator=g, device=dev)
    sd = builder.build_index(base, centres, lab, seed=20261207, device=dev)
    del base
    torch.cuda.empty_cache()
    return sd, q.cpu().numpy()


def _search(cb, sd, q):
    e = cb.HybridIndex(0)
    e.load_search_data(sd)
    e.prepare_workspace(NQ, K, NPROBE)
    e.reset_buffer(q)
    d, i = e.search(q, K, NPROBE)
    return e, d, i


def test_fullsize_properties_and_oracle_sample(fullsize):
    import coraanns_b200 as cb
    sd, q = fullsize
    e, d, i = _search(cb, sd, q)
    assert np.isfinite(d).all()                      # >= k candidates for every query
    dd = d[:, 1:] - d[:, :-1]                        # ascending (distance, id)
    assert ((dd > 0) | ((dd == 0) & (i[:, 1:] > i[:, :-1]))).all()
    assert (np.sort(i, axis=1)[:, 1:] != np.sort(i, axis=1)[:, :-1]).all()  # unique ids
    t = e.capture_thresholds(NQ)
    assert t.tobytes() == d[:, K - 1].copy().tobytes()
    # a second search of the same batch returns the same bytes
    d2, i2 = e.search(q, K, NPROBE)
    assert d2.tobytes() == d.tobytes() and np.array_equal(i2, i)
    cand = e.debug("cand_count", NQ)
    e.close()
    # bit-exact against the oracle on a seeded sample
    rng = np.random.default_rng(5)
    sample = np.sort(rng.choice(NQ, 48, replace=False))
    ref = po.OracleIndex(sd).search(q[sample], K, NPROBE, with_details=True)
    assert np.array_equal(i[sample], ref["ids"])
    assert d[sample].tobytes() == ref["dist"].tobytes()
    assert np.array_equal(cand[sample].astype(np.uint64), ref["cand_count"])


def test_fullsize_two_shards_equal_whole(fullsize):
    import torch
    import coraanns_b200 as cb
    from coraanns_b200.shard import exchange_words
    sd, q = fullsize
    e, want_d, want_i = _search(cb, sd, q)
    e.close()
    engines = []
    for r in range(2):
        s = cb.HybridIndex(0)
        s.shard_configure(r, 2)
        s.load_search_data(sd)
        s.prepare_workspace(NQ, K, NPROBE)
        engines.append(s)
    w = exchange_words(NQ, K)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        dq = torch.from_numpy(q).cuda()
        sends = [torch.empty(w, dtype=torch.int64, device="cuda") for _ in range(2)]
        recv = torch.empty(2 * w, dtype=torch.int64, device="cuda")
        od = torch.empty((NQ, K), dtype=torch.float32, device="cuda")
        oi = torch.empty((NQ, K), dtype=torch.int32, device="cuda")
        for s, b in zip(engines, sends):
            s.shard_search_begin(dq.data_ptr(), NQ, K, NPROBE, b.data_ptr(), st.cuda_stream)
        torch.cat(sends, out=recv)
        for s, b in zip(engines, sends):
            s.shard_search_resume(recv.data_ptr(), b.data_ptr())
        torch.cat(sends, out=recv)
        engines[0].shard_search_end(recv.data_ptr(), od.data_ptr(), oi.data_ptr())
    st.synchronize()
    for s in engines:
        s.check_device()
        s.close()
    assert np.array_equal(oi.cpu().numpy().view(np.uint32), want_i)
    assert od.cpu().numpy().tobytes() == want_d.tobytes()
