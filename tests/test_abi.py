"""libkvs_b200.so loads without a GPU, exports every symbol include/kvs_b200.h declares,
and its struct layouts match the ctypes binding.  No kernel is launched."""

import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _declared_functions():
    text = (REPO / "include" / "kvs_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvs_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from kvstreams import _native as N

    return N.load_library()


def test_library_is_in_tree(lib):
    from kvstreams import _native as N

    assert N.LIB_PATH.exists()
    assert N.LIB_PATH.is_relative_to(REPO)


def test_every_declared_symbol_is_exported(lib):
    names = _declared_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n
    from kvstreams import _native as N

    assert set(names) == set(N.SIGNATURES), set(names) ^ set(N.SIGNATURES)


def test_struct_layouts_match(lib):
    import ctypes as C

    from kvstreams import _native as N

    for which, st in N.STRUCTS.items():
        assert lib.kvs_abi_struct_size(which) == C.sizeof(st)
    assert lib.kvs_abi_version() == 4


def test_host_only_size_queries(lib):
    # pure host arithmetic: no device needed
    assert lib.kvs_evict_scratch_bytes(256, 512) >= 256 * 512 * 5
    assert lib.kvs_check_scratch_bytes(200000) >= 200000 // 8
    assert lib.kvs_replay_scratch_bytes(16, 32768) >= 0


def test_null_arguments_are_rejected_before_launch(lib):
    # argument validation returns KVS_E_ARG without touching CUDA
    assert lib.kvs_append_slots(None, None, None, None, None, None) == -1
    assert lib.kvs_replay_attention(None, None) == -1
    assert lib.kvs_rope(None, 0, None, 0, 1, 2, None, None) == -1


def test_noalloc_limits_are_checked_on_the_host(lib):
    """kvs_evict_positions_noalloc refuses a batch beyond its built-in scratch -- more than 256
    sequences, or tables longer than 1024 entries -- with KVS_E_NOALLOC_LIMIT before any CUDA
    call, and an empty batch is a no-op (struct pointers are never dereferenced on the device
    here: nothing may be launched)."""
    import ctypes as C

    from kvstreams import _native as N

    cache = N.KvsCache(n_layers=1, num_blocks=4096, block_size=16, n_kv_heads=1, head_dim=2, max_seqs=512,
                       max_blocks=1024, dtype=N.KVS_F32)
    for num_seqs, max_blocks, want in ((257, 1024, -5), (1, 1025, -5), (0, 1024, 0)):
        cache.max_blocks = max_blocks
        batch = N.KvsBatch(seq_slots=None, cu_tokens=None, num_seqs=num_seqs, total_tokens=num_seqs)
        rc = lib.kvs_evict_positions_noalloc(C.byref(cache), C.byref(batch), None, None, None, None, None, 1, None)
        assert rc == want, (num_seqs, max_blocks, rc)
