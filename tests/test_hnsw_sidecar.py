"""Indexes whose centroids live in an hnswlib sidecar (`<index>.hnsw`, the reference's layout
for nlist >= 20000: ivf.hpp:312, initializer.hpp:252-279).

The fixture rewrites a golden flat index without its embedded centroids and writes the
sidecar in the layout hnswlib's saveIndex produces (hnswalg.h:685-713): a 96-byte header,
one level-0 record per element (links, the D-float vector at offsetData, the u64 label at
label_offset), then the upper-level link lists. Element order is shuffled, since the
labels, not the positions, name the clusters. The Python reader (CPU) and the engine's
loader (GPU) must recover the flat index's centroids and search results.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

import py_oracle as po
from conftest import GOLDEN


def write_hnsw_split(flat_path, out_path, seed=0):
    """Copy of `flat_path` with its centroids moved to an hnswlib-layout sidecar."""
    raw = flat_path.read_bytes()
    ivf = po.read_ivf_file(flat_path)
    nlist, D, dim = int(ivf["nlist"]), int(ivf["D"]), int(ivf["dim"])
    head = 34 + 8 * nlist + 4 * dim * D
    out_path.write_bytes(raw[:head] + raw[head + 4 * D * nlist:])
    rng = np.random.default_rng(seed)
    M0 = 32
    links = 4 + 4 * M0                       # link-list count + neighbour ids
    data_off, label_off = links, links + 4 * D
    per = label_off + 8
    order = rng.permutation(nlist)           # element i holds cluster order[i]
    hdr = struct.pack("<6Q iI 3Q d Q", 0, nlist, nlist, per, label_off, data_off, 1, 0,
                      16, M0, 16, 1.0 / np.log(16), 200)
    level0 = np.zeros((nlist, per), np.uint8)
    level0[:, :links] = rng.integers(0, 256, (nlist, links), dtype=np.uint8)
    level0[:, data_off:label_off] = ivf["centroids"][order].view(np.uint8).reshape(nlist, -1)
    level0[:, label_off:] = order.astype(np.uint64).view(np.uint8).reshape(nlist, 8)
    tail = bytearray()
    for i in range(nlist):                   # upper levels: a few elements have one
        size = 4 * (16 + 1) if i % 7 == 0 else 0
        tail += struct.pack("<I", size) + bytes(rng.integers(0, 256, size, dtype=np.uint8))
    (out_path.parent / (out_path.name + ".hnsw")).write_bytes(hdr + level0.tobytes() + bytes(tail))
    return ivf


@pytest.mark.parametrize("name", ["demo", "d96"])
def test_python_reader_recovers_sidecar_centroids(tmp_path, name):
    flat = GOLDEN / f"{name}.index"
    split = tmp_path / f"{name}.index"
    ref = write_hnsw_split(flat, split)
    got = po.read_ivf_file(split)
    assert np.array_equal(got["centroids"], ref["centroids"])
    for key in ("sizes", "rotator", "ids"):
        assert np.array_equal(got[key], ref[key])
    assert np.array_equal(np.asarray(got["batch"]), np.asarray(ref["batch"]))
    assert np.array_equal(np.asarray(got["ex"]), np.asarray(ref["ex"]))


def test_sidecar_labels_must_name_every_cluster(tmp_path):
    split = tmp_path / "demo.index"
    write_hnsw_split(GOLDEN / "demo.index", split)
    side = tmp_path / "demo.index.hnsw"
    raw = bytearray(side.read_bytes())
    hdr = struct.unpack_from("<6Q", raw, 0)
    per, label_off = hdr[3], hdr[4]
    struct.pack_into("<Q", raw, 96 + label_off, 10 ** 6)  # element 0: no such cluster
    side.write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        po.read_ivf_file(split)


@pytest.mark.gpu
def test_engine_loads_sidecar_index(tmp_path):
    import coraanns_b200 as cb
    split = tmp_path / "d96.index"
    write_hnsw_split(GOLDEN / "d96.index", split)
    z = np.load(GOLDEN / "d96.npz")
    q = z["queries"]
    out = []
    for path in (GOLDEN / "d96.index", split):
        e = cb.HybridIndex(0)
        e.load_index_file(str(path))
        e.prepare_workspace(len(q), 10, 6)
        e.reset_buffer(q)
        out.append(e.search(q, 10, 6))
        e.close()
    assert out[0][0].tobytes() == out[1][0].tobytes()
    assert np.array_equal(out[0][1], out[1][1])
