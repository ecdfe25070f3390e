"""CPU tests of the C ABI boundary: the library loads and exports every declared symbol.

No compute call is made (there may be no GPU here)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "cora_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cora_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import coraanns_b200 as cb
    lib = ctypes.CDLL(str(cb.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(cb.EXPORTS) == names


def test_library_targets_sm100a_only():
    """The build recipe compiles for sm_100a and nothing else."""
    mk = (ROOT / "cgcl-coraanns_b200" / "Makefile").read_text()
    assert "arch=compute_100a,code=sm_100a" in mk
    assert "sm_90" not in mk and "sm_80" not in mk


def test_last_error_is_empty_string_initially():
    import coraanns_b200 as cb
    assert isinstance(cb._lib.cora_last_error(), bytes)


def test_null_engine_calls_are_rejected_without_a_gpu():
    """Null handles are rejected by the boundary itself (no device work)."""
    import coraanns_b200 as cb
    rc = cb._lib.cora_prepare_workspace(None, 1, 1, 1)
    assert rc == cb.CORA_EINVAL
    assert b"null engine" in cb._lib.cora_last_error()
    assert cb._lib.cora_get_vanguard_size(None) == 0


def test_shard_entry_points_reject_null_engines_and_size_probe_buffers():
    """The shard-local load and the split-probing calls validate their handle before any
    device work; the probe exchange holds ceil(nq / world) * nprobe words + a status word."""
    import coraanns_b200 as cb
    L = cb._lib
    z = [None] * 9
    assert L.cora_load_shard_arrays(None, 1, 64, 64, 1, 7, *z) == cb.CORA_EINVAL
    assert L.cora_shard_search_probe(None, None, 1, 1, 1, None, None) == cb.CORA_EINVAL
    assert L.cora_shard_search_begin_probed(None, None, None) == cb.CORA_EINVAL
    assert L.cora_shard_probe_words(10_000, 8, 3) == 3334 * 8 + 1
    assert L.cora_shard_probe_words(5, 4, 8) == 1 * 4 + 1
    assert L.cora_shard_probe_words(5, 4, 0) == 0
