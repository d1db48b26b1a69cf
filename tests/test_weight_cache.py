"""Weight commitment cache in the engine's SWCF file format (weight_cache.rs): byte layout,
round trip, older versions, fingerprint, model-id check, and root caching."""
import struct

import numpy as np
import pytest

from zkml_b200.weight_cache import (CachedWeight, WeightCommitmentCache, compute_weight_fingerprint)


def test_file_layout_of_one_root_entry(tmp_path):
    c = WeightCommitmentCache("qwen", bytes(range(32)))
    c.insert_root(7, 8, 16, 0x1234)
    p = tmp_path / "c.swcf"
    c.save(str(p))
    want = (b"SWCF" + struct.pack("<I", 4) + struct.pack("<I", 4) + b"qwen" + bytes(range(32)) +
            struct.pack("<I", 1) + struct.pack("<4Q", 7, 0, 8, 16) + struct.pack("<I", 0) + bytes(32) +
            struct.pack("<I", 0) + b"\x01" + (0x1234).to_bytes(32, "big") + b"\x00")
    assert p.read_bytes() == want


def test_round_trip_and_lookups(tmp_path):
    c = WeightCommitmentCache("m")
    fb = np.arange(12, dtype=np.uint32).reshape(3, 4)
    rj = np.arange(8, dtype=np.uint32).reshape(2, 4) + 100
    c.insert(3, 64, 8192, 16384, CachedWeight(fb, 0xABC, rj, 0xDEF, "/tmp/tree"))
    c.insert_root(5, 4096, 8192, 2**250 + 1)
    p = str(tmp_path / "c.swcf")
    c.save(p)
    d = WeightCommitmentCache.load(p)
    e = d.get(3, 64, 8192, 16384)
    assert (e.f_b == fb).all() and (e.r_j == rj).all() and e.b_commitment == 0xABC
    assert e.initial_mle_root == 0xDEF and e.merkle_tree_cache_path == "/tmp/tree"
    assert d.get_root(5, 4096, 8192) == 2**250 + 1 and d.get_root(5, 4096, 4096) is None
    assert len(d) == 2 and not d.dirty and d.auto_save_path == p


def test_reads_version_1(tmp_path):
    b = (b"SWCF" + struct.pack("<I", 1) + struct.pack("<I", 1) + b"x" + struct.pack("<I", 1) +
         struct.pack("<4Q", 1, 2, 4, 8) + struct.pack("<I", 1) + struct.pack("<4I", 1, 2, 3, 4) +
         (99).to_bytes(32, "big") + struct.pack("<I", 0))
    p = tmp_path / "v1.swcf"
    p.write_bytes(b)
    d = WeightCommitmentCache.load(str(p))
    assert d.fingerprint == bytes(32) and d.get(1, 2, 4, 8).b_commitment == 99
    assert d.get(1, 2, 4, 8).initial_mle_root is None


def test_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.swcf"
    p.write_bytes(b"NOPE" + bytes(8))
    with pytest.raises(ValueError):
        WeightCommitmentCache.load(str(p))
    p.write_bytes(b"SWCF" + struct.pack("<I", 9))
    with pytest.raises(ValueError):
        WeightCommitmentCache.load(str(p))
    c = WeightCommitmentCache.load_or_new(str(p), "m")
    assert len(c) == 0 and c.auto_save_path == str(p)


def test_load_or_new_checks_model_id(tmp_path):
    p = str(tmp_path / "c.swcf")
    c = WeightCommitmentCache("a")
    c.insert_root(1, 2, 2, 5)
    c.save(p)
    assert len(WeightCommitmentCache.load_or_new(p, "a")) == 1
    assert len(WeightCommitmentCache.load_or_new(p, "b")) == 0


def fingerprint_spec(weights):
    M = (1 << 64) - 1
    s = [0xCBF29CE484222325] * 4
    P = 0x100000001B3
    for nid, w in weights:
        d = np.asarray(w).reshape(-1)
        n = d.size
        s[0] = ((s[0] * P) & M) ^ nid
        s[1] = ((s[1] * P) & M) ^ w.shape[0]
        s[2] = ((s[2] * P) & M) ^ w.shape[1]
        s[3] = ((s[3] * P) & M) ^ n
        step = max(1, n // 8)
        for i in range(min(8, n)):
            s[i % 4] = ((s[i % 4] * P) & M) ^ int(d[min(i * step, n - 1)])
    return b"".join(x.to_bytes(8, "little") for x in s)


def test_fingerprint_follows_the_definition_and_detects_changes():
    rng = np.random.default_rng(0)
    ws = [(0, rng.integers(0, 2**31 - 1, (64, 48), dtype=np.uint32)), (2, rng.integers(0, 127, (3, 5),
                                                                                        dtype=np.uint32))]
    fp = compute_weight_fingerprint(ws)
    assert fp == fingerprint_spec(ws)
    c = WeightCommitmentCache("m", fp)
    assert c.validate_fingerprint(ws)
    w0 = ws[0][1].copy()
    w0.flat[0] ^= 1  # a sampled element
    assert not c.validate_fingerprint([(0, w0), ws[1]])
    w0 = ws[0][1].copy()
    w0.flat[1] ^= 1  # not sampled
    assert c.validate_fingerprint([(0, w0), ws[1]])
    assert WeightCommitmentCache("m").validate_fingerprint([(0, w0)])


def test_root_for_commits_once():
    calls = []
    c = WeightCommitmentCache("m")
    w = np.ones((5, 9), np.uint32)
    for _ in range(3):
        assert c.root_for(4, w, lambda x: calls.append(1) or 77) == 77
    assert len(calls) == 1 and c.get_root(4, 8, 16) == 77
