"""The C ABI without a GPU: the library loads, exports every symbol include/vdbgpu.h declares,
reads the reference's index files (CRC32C framing) and fails loudly instead of falling back."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from helpers import golden

HEADER = os.path.join(ROOT, "include", "vdbgpu.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"VDBGPU_API\s+[\w\s\*]+?\b(vdbgpu_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import vdb_b200
    lib = ctypes.CDLL(vdb_b200.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 14
    for s in syms:
        assert hasattr(lib, s), s
    # The Python host binds exactly the declared surface.
    assert sorted(vdb_b200._SIGNATURES) == syms
    assert vdb_b200.lib().vdbgpu_abi_version() == 1


def test_index_files_are_checked():
    import vdb_b200
    for name, t in (("flat_int", "flat_file"), ("hnsw", "index_file"), ("hnsw_sq8", "index_file"),
                    ("ivfpq", "index_file"), ("pqflat", "index_file")):
        data = bytes(golden(name)[t])
        want = {"flat_int": 0, "hnsw": 1, "hnsw_sq8": 2, "pqflat": 3, "ivfpq": 4}[name]
        assert vdb_b200.inspect_index_file(data) == want
        # A flipped byte is caught by the CRC footer (tests/hnsw_test.cc:108-111) and a truncated
        # file is rejected (tests/index_test.cc:64).
        bad = bytearray(data)
        bad[len(bad) // 2] ^= 0x5A
        with pytest.raises(vdb_b200.VdbError) as e:
            vdb_b200.inspect_index_file(bytes(bad))
        assert e.value.code == 5  # Corruption
        with pytest.raises(vdb_b200.VdbError):
            vdb_b200.inspect_index_file(data[:-1])


def test_no_gpu_means_an_error_not_a_fallback():
    import vdb_b200
    if vdb_b200.device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(vdb_b200.VdbError) as e:
        vdb_b200.Context(0)
    assert e.value.code == vdb_b200.UNAVAILABLE


def test_bitset_packing_matches_reference_layout():
    import vdb_b200
    rng = np.random.default_rng(3)
    mask = rng.random(1000) < 0.3
    words = vdb_b200.pack_bitset(mask)
    assert words.dtype == np.uint64 and words.size == (1000 + 63) // 64
    for r in range(1000):
        assert bool((int(words[r >> 6]) >> (r & 63)) & 1) == mask[r]
    np.testing.assert_array_equal(vdb_b200.unpack_bitset(words, 1000), mask)
