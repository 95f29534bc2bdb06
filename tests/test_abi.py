"""CPU tests of the C ABI library: it loads, exports every declared entry
point, and its host-side prefix-cache logic matches the reference's tests
(Tests/NovaMLXPrefixCacheTests/PrefixCacheTests.swift) and the golden hashes.
No CUDA compute is called here."""
import json
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "novamlx_b200" / "libnovamlx_cuda.so"
KAT = json.loads((Path(__file__).parent / "golden" / "kat.json").read_text())


def declared_symbols():
    text = (ROOT / "include" / "nmx.h").read_text()
    return sorted(set(re.findall(r"NMX_API[^;(]*?\b(nmx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    assert LIB.exists(), "build the library first (python -m novamlx_b200.build)"
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (nmx_[a-z0-9_]+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    assert len(declared_symbols()) >= 40


def test_library_is_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", str(LIB)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    archs = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert archs == {"100a"}, archs


@pytest.fixture(scope="module")
def nmx():
    from novamlx_b200 import nmx as mod
    return mod


def test_version(nmx):
    assert "sm_100a" in nmx.version()


@pytest.mark.parametrize("case", KAT["block_hash"], ids=lambda c: c["hex"][:8])
def test_block_hash_golden(nmx, case):
    parent = bytes.fromhex(case["parent"]) if case["parent"] else None
    got = nmx.BlockHasher.compute_block_hash(parent, case["tokens"], case["model"])
    assert got.hex() == case["hex"]


def test_chain_hashes_golden(nmx):
    c = KAT["chain"]
    got = nmx.BlockHasher.compute_chain_hashes(c["tokens"], c["block_size"], c["model"])
    assert [h.hex() for h in got] == c["hex"]


# ---- PrefixCacheTests.swift, restated ------------------------------------

def test_hasher_consistency(nmx):
    H = nmx.BlockHasher
    t = [1, 2, 3, 4, 5, 6, 7, 8]
    assert H.compute_block_hash(None, t, "test-model") == H.compute_block_hash(None, t, "test-model")


def test_hasher_difference(nmx):
    H = nmx.BlockHasher
    assert H.compute_block_hash(None, [1, 2, 3], "test") != H.compute_block_hash(None, [4, 5, 6], "test")


def test_hasher_chain_depends_on_parent(nmx):
    H = nmx.BlockHasher
    pa = H.compute_block_hash(None, [10, 20], "test")
    pb = H.compute_block_hash(None, [30, 40], "test")
    assert H.compute_block_hash(pa, [1, 2, 3], "test") != H.compute_block_hash(pb, [1, 2, 3], "test")


def test_chain_count(nmx):
    H = nmx.BlockHasher
    assert len(H.compute_chain_hashes(list(range(256)), 64, "test")) == 4
    assert H.compute_chain_hashes(list(range(32)), 64, "test") == []


def test_model_isolation(nmx):
    H = nmx.BlockHasher
    assert H.compute_block_hash(None, [1, 2, 3], "model-a") != H.compute_block_hash(None, [1, 2, 3], "model-b")


def test_pool_allocate_free(nmx):
    p = nmx.PagedBlockPool(64, 100, 10, "test")
    b = p.allocate_block()
    assert b is not None and p.ref_count(b) == 1
    assert p.get_stats()[:3] == (10, 1, 8)


def test_pool_no_match(nmx):
    p = nmx.PagedBlockPool(64, 100, 10, "test")
    assert p.find_shared_prefix(list(range(128))) == ([], 128)


def test_pool_register_and_find(nmx):
    p = nmx.PagedBlockPool(4, 100, 10, "test")
    b = p.allocate_block()
    p.register_block(b, [0, 1, 2, 3], None)
    ids, rem = p.find_shared_prefix(list(range(8)))
    assert ids == [b] and rem == 4


def test_pool_refcount(nmx):
    p = nmx.PagedBlockPool(4, 100, 10, "test")
    b = p.allocate_block()
    p.increment_ref(b)
    assert p.ref_count(b) == 2
    assert p.get_stats()[3] == 1
    p.free_block(b)
    assert p.ref_count(b) == 1
    p.free_block(b)
    assert p.get_stats()[2] == 9


def test_pool_fork_table(nmx):
    p = nmx.PagedBlockPool(4, 100, 10, "test")
    b = p.allocate_block()
    p.create_block_table("req-1")
    p.append_block("req-1", b)
    p.fork_block_table("req-1", "req-2")
    assert p.ref_count(b) == 2
    assert p.block_table("req-2") == [b]
    p.delete_block_table("req-1")
    assert p.ref_count(b) == 1


def test_pool_clear(nmx):
    p = nmx.PagedBlockPool(4, 100, 10, "test")
    p.allocate_block()
    p.allocate_block()
    p.clear()
    t, _, f, _ = p.get_stats()
    assert (t, f) == (10, 9)


def test_pool_fifo_and_growth(nmx):
    p = nmx.PagedBlockPool(4, 300, 10, "test")
    ids = [p.allocate_block() for _ in range(9)]
    assert ids == list(range(1, 10))  # block 0 is the null block
    assert p.allocate_block() == 10  # grew by min(256, 300 - 10)
    assert p.get_stats()[0] == 266
    p.free_block(3)
    p.free_block(5)
    # free list is FIFO: freed blocks go to the tail
    nxt = [p.allocate_block() for _ in range(257)]  # 11..265, then 3, 5
    assert nxt[-3:] == [265, 3, 5]
    assert p.allocate_block() == 266  # grows again (max 300)


def test_pool_exhaustion(nmx):
    p = nmx.PagedBlockPool(4, 3, 3, "test")
    assert [p.allocate_block() for _ in range(3)] == [1, 2, None]


def test_pool_freed_block_hash_quirk(nmx):
    """Freeing drops the map entry; re-allocating the freed block drops the
    entry again (PagedBlockPool.swift:146-149,169-172)."""
    p = nmx.PagedBlockPool(4, 3, 3, "test")
    a = p.allocate_block()
    p.register_block(a, [1, 2, 3, 4], None)
    p.free_block(a)
    assert p.find_shared_prefix([1, 2, 3, 4]) == ([], 4)
    b = p.allocate_block()
    p.register_block(b, [1, 2, 3, 4], None)
    assert p.find_shared_prefix([1, 2, 3, 4]) == ([b], 0)
    c = p.allocate_block()  # this is `a` again (FIFO), still carrying the old hash
    assert c == a
    assert p.find_shared_prefix([1, 2, 3, 4]) == ([], 4)


def test_prefix_chain_longest_match(nmx):
    p = nmx.PagedBlockPool(16, 1000, 100, "llama")
    toks = list(range(1000, 1064))
    parent = None
    ids = []
    for i in range(3):
        b = p.allocate_block()
        p.register_block(b, toks[16 * i:16 * (i + 1)], parent)
        parent = nmx.BlockHasher.compute_block_hash(parent, toks[16 * i:16 * (i + 1)], "llama")
        ids.append(b)
    got, rem = p.find_shared_prefix(toks + [7] * 5)
    assert got == ids and rem == 69 - 48
    # a different first block breaks the chain entirely
    assert p.find_shared_prefix([0] + toks[1:])[0] == []
