"""ctypes binding of libkvs_b200.so (the C ABI declared in include/kvs_b200.h).

The library is built in-tree by ``faster-rl-training_b200/csrc/build.py``.  There is
no fallback: if the library or a CUDA device is missing, :func:`lib` raises.
Struct layouts are checked against ``kvs_abi_struct_size`` when the library loads.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_NAME = "libkvs_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

KVS_F32, KVS_F64, KVS_BF16, KVS_F16 = 0, 1, 2, 3
DTYPE_CODE = {torch.float32: KVS_F32, torch.float64: KVS_F64, torch.bfloat16: KVS_BF16, torch.float16: KVS_F16}

# device status codes (enum kvs_status)
ST_OK = 0
ST_OUT_OF_BLOCKS = 1
ST_DOUBLE_FREE = 2
ST_NOT_FULL_BLOCK = 3
ST_TABLE_OVERFLOW = 4
ST_TRUNCATE = 5
ST_INV_DUP_BLOCK = 6
ST_INV_TABLE_LEN = 7
ST_INV_HOLE = 8
ST_INV_ORDER = 9
ST_SPAN_CAPACITY = 10
ST_OWNER = 11
ST_KERNEL_TIMEOUT = 12
ST_SEQ_TOO_LONG = 13
ST_LOG_CAPACITY = 14

# device compaction (kvs_segments / kvs_compact)
POLICY_CODES = {"keep_recent": 0, "markovian": 1, "summary": 2, "token_window": 3}
EV_FIELDS = 9  # KVS_EV_TIME .. KVS_EV_SEG_OFFSET

RC_NAMES = {-1: "bad argument", -2: "unsupported shape/dtype", -3: "CUDA launch error", -4: "scratch too small",
            -5: "request exceeds the built-in scratch of a no-alloc entry point"}

STAT_FIELDS = (
    "written_tokens",
    "evicted_tokens",
    "evicted_blocks",
    "truncated_tokens",
    "peak_blocks",
    "eviction_calls",
    "shrunk_tokens",
)
STAT_COUNT = 8
STATUS_WORDS = 4
ABI_VERSION = 4  # KVS_ABI_VERSION of include/kvs_b200.h
NEVER = (1 << 63) - 1


class KvsCache(C.Structure):
    _fields_ = [
        ("k", C.c_void_p),
        ("v", C.c_void_p),
        ("slot_pos", C.c_void_p),
        ("tables", C.c_void_p),
        ("n_blocks", C.c_void_p),
        ("lengths", C.c_void_p),
        ("free_stack", C.c_void_p),
        ("free_top", C.c_void_p),
        ("block_owner", C.c_void_p),
        ("stats", C.c_void_p),
        ("status", C.c_void_p),
        ("n_layers", C.c_int32),
        ("num_blocks", C.c_int32),
        ("block_size", C.c_int32),
        ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("max_seqs", C.c_int32),
        ("max_blocks", C.c_int32),
        ("dtype", C.c_int32),
    ]


class KvsBatch(C.Structure):
    _fields_ = [
        ("seq_slots", C.c_void_p),
        ("cu_tokens", C.c_void_p),
        ("num_seqs", C.c_int32),
        ("total_tokens", C.c_int32),
    ]


class KvsDecodeArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p),
        ("k_new", C.c_void_p),
        ("v_new", C.c_void_p),
        ("positions", C.c_void_p),
        ("slot_blocks", C.c_void_p),
        ("slot_offsets", C.c_void_p),
        ("inv_freq", C.c_void_p),
        ("out", C.c_void_p),
        ("scratch", C.c_void_p),
        ("scratch_bytes", C.c_size_t),
        ("scale", C.c_double),
        ("layer", C.c_int32),
        ("n_heads", C.c_int32),
        ("grid_ctas", C.c_int32),
        ("tail_singles", C.c_int32),
        ("q_stride", C.c_int64),
        ("kv_stride", C.c_int64),
        ("plan", C.c_int32),
    ]


PLAN_NONE, PLAN_BUILD, PLAN_REUSE = 0, 1, 2  # kvs_decode_plan


class KvsReplayArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p),
        ("k", C.c_void_p),
        ("v", C.c_void_p),
        ("evicted_at", C.c_void_p),
        ("lengths", C.c_void_p),
        ("out", C.c_void_p),
        ("scratch", C.c_void_p),
        ("scratch_bytes", C.c_size_t),
        ("batch", C.c_int32),
        ("seq_len", C.c_int32),
        ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("dtype", C.c_int32),
        ("scale", C.c_double),
        ("flags", C.c_int32),
        ("reserved", C.c_int32),
        ("row_lse", C.c_void_p),
    ]


_P = C.c_void_p
_I = C.c_int32
_Z = C.c_size_t

# name -> (restype, argtypes); every symbol of include/kvs_b200.h
class KvsSegments(C.Structure):
    _fields_ = [
        ("start", C.c_void_p),
        ("end", C.c_void_p),
        ("evicted_at", C.c_void_p),
        ("flags", C.c_void_p),
        ("count", C.c_void_p),
        ("ev_count", C.c_void_p),
        ("ev_meta", C.c_void_p),
        ("ev_spans", C.c_void_p),
        ("ev_segs", C.c_void_p),
        ("ev_fill", C.c_void_p),
        ("stats", C.c_void_p),
        ("max_seqs", C.c_int32),
        ("max_segs", C.c_int32),
        ("max_events", C.c_int32),
        ("span_pool", C.c_int32),
        ("seg_pool", C.c_int32),
        ("reserved", C.c_int32),
    ]


SIGNATURES = {
    "kvs_abi_struct_size": (_Z, [C.c_int]),
    "kvs_abi_version": (C.c_int, []),
    "kvs_device_sm_count": (C.c_int, []),
    "kvs_launch_count": (C.c_longlong, []),
    "kvs_cache_reset": (C.c_int, [_P, _P]),
    "kvs_append_slots": (C.c_int, [_P, _P, _P, _P, _P, _P]),
    "kvs_write_kv": (C.c_int, [_P, _I, _P, _P, _P, _P, _I, _P]),
    "kvs_evict_scratch_bytes": (_Z, [_I, _I]),
    "kvs_evict_positions": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _Z, _P]),
    "kvs_evict_positions_noalloc": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I, _P]),
    "kvs_evict_blocks": (C.c_int, [_P, _P, _P, _P, _Z, _P]),
    "kvs_release": (C.c_int, [_P, _P, _P, _I, _P]),
    "kvs_check_scratch_bytes": (_Z, [_I]),
    "kvs_check_invariants": (C.c_int, [_P, _P, _P, _P, _Z, _P]),
    "kvs_rope": (C.c_int, [_P, _I, _P, _I, _I, _I, _P, _P]),
    "kvs_rope_copy": (C.c_int, [_P, C.c_int64, _P, C.c_int64, _I, _P, _I, _I, _I, _P, _P]),
    "kvs_paged_attention": (C.c_int, [_P, _P, _I, _P, _P, _I, C.c_double, _P]),
    "kvs_decode_scratch_bytes": (_Z, [_P, _I, _I, _I]),
    "kvs_paged_decode": (C.c_int, [_P, _P, _P, _P]),
    "kvs_paged_decode_path": (C.c_int, [_P, _P, _P]),
    "kvs_evicted_at": (C.c_int, [_P, _P, _P, _P, _P, _I, _I, _P, _P]),
    "kvs_replay_scratch_bytes": (_Z, [_I, _I]),
    "kvs_replay_attention": (C.c_int, [_P, _P]),
    "kvs_replay_backward_scratch_bytes": (_Z, [_I, _I, _I, _I]),
    "kvs_replay_attention_backward": (C.c_int, [_P, _P, _P, _P, _P, _P]),
    "kvs_replay_backward_path": (C.c_int, [_P, _P]),
    "kvs_compact_plan": (C.c_int, [_P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "kvs_compact_scratch_bytes": (_Z, [_P, _P, _I]),
    "kvs_compact": (C.c_int, [_P, _P, _P, _I, _I, _I, _P, _P, _Z, _P]),
    "kvs_lse_gather": (C.c_int, [_P, C.c_int64, _I, _I, _P, C.c_double, _I, _P, _P, _P]),
    "kvs_sample": (C.c_int, [_P, C.c_int64, _I, _I, C.c_double, _I, _I, C.c_uint64, C.c_uint64, _P, _P, _P]),
    "kvs_rms_norm": (C.c_int, [_P, _P, _P, _P, C.c_int64, _I, C.c_int64, C.c_int64, C.c_double, _I, _P]),
    "kvs_rms_norm_backward_scratch_bytes": (C.c_size_t, [C.c_int64, _I]),
    "kvs_rms_norm_backward": (C.c_int, [_P, _P, _P, _P, _P, _P, C.c_int64, _I, C.c_int64, C.c_int64, C.c_int64, _I, _P,
                                        C.c_size_t, _P]),
    "kvs_silu_mul": (C.c_int, [_P, _P, C.c_int64, _I, C.c_int64, C.c_int64, _I, _P]),
    "kvs_silu_mul_backward": (C.c_int, [_P, _P, _P, C.c_int64, _I, C.c_int64, C.c_int64, C.c_int64, _I, _P]),
    "kvs_lse_gather_backward": (C.c_int, [_P, C.c_int64, _I, _I, _P, _P, _P, C.c_double, _I, _P, C.c_int64, _I, _P]),
    "kvs_selftest_umma": (C.c_int, [_P, _P, _P, _I, _P, _P]),
    "kvs_selftest_wait": (C.c_int, [_I, C.c_uint32, _P, _P]),
    "kvs_lm_head_logprobs_scratch_bytes": (_Z, [_I, _I]),
    "kvs_lm_head_logprobs_supported": (C.c_int, [_I]),
    "kvs_lm_head_logprobs": (C.c_int, [_P, C.c_int64, _P, C.c_int64, _I, _I, _I, _P, C.c_double, _P, _P, _P, _Z,
                                       _P]),
}

STRUCTS = {0: KvsCache, 1: KvsBatch, 2: KvsDecodeArgs, 3: KvsReplayArgs, 4: KvsSegments}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def load_library(path: Path | str | None = None) -> C.CDLL:
    """Load the shared library (no GPU needed) and check the struct layouts."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path or os.environ.get("KVS_B200_LIB", LIB_PATH))
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build the kvstreams CUDA library first "
                "(python faster-rl-training_b200/csrc/build.py); there is no CPU fallback"
            )
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        for which, st in STRUCTS.items():
            got = lib.kvs_abi_struct_size(which)
            if got != C.sizeof(st):
                raise RuntimeError(f"ABI mismatch for {st.__name__}: library {got} B, binding {C.sizeof(st)} B")
        if lib.kvs_abi_version() != ABI_VERSION:
            raise RuntimeError(f"library ABI version {lib.kvs_abi_version()}, binding {ABI_VERSION}: rebuild it")
        _lib = lib
        return lib


def lib() -> C.CDLL:
    """The library, for a call that launches kernels: requires a CUDA device."""
    if not torch.cuda.is_available():
        raise RuntimeError("kvstreams kernels need a CUDA (sm_100a) device; none is visible")
    return load_library()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {RC_NAMES.get(rc, rc)} (rc={rc})")


def to_device(values, dtype: torch.dtype, device) -> torch.Tensor:
    """A host list or array as a tensor on ``device`` without waiting for the GPU: staged in pinned
    memory and copied on the current stream (a copy from pageable memory, as
    ``torch.tensor(values, device="cuda")`` makes, first waits for the stream's queued work)."""
    t = torch.as_tensor(values, dtype=dtype)
    dev = torch.device(device)
    if dev.type != "cuda":
        return t.to(dev)
    return t.pin_memory().to(dev, non_blocking=True)


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must live on a CUDA device (got {t.device}); there is no CPU path")
