"""ctypes bindings of libkvs_b200.so, the C ABI declared in include/kvs.h.

This module is the Python side of the drop-in boundary. The reference binds its C++ classes with
nanobind (src/python/bindings.cpp); here the product library exports a plain C ABI and this
module declares every entry point once. Loading fails loudly when the library is missing: there is
no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_NAME = "libkvs_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

KVS_ABI_VERSION = 1

OK = 0
E_INVAL = -1
E_CUDA = -2
E_NOSPACE = -3
E_TIMEOUT = -4
E_TOO_SMALL = -5
E_QUARANTINED = -6
E_CLOSED = -7
E_FORMAT = -8

LOC_DEVICE, LOC_HOST, LOC_PENDING, LOC_ABSENT = 0, 1, 2, -1

_ERROR_NAMES = {
    E_INVAL: "KVS_E_INVAL",
    E_CUDA: "KVS_E_CUDA",
    E_NOSPACE: "KVS_E_NOSPACE",
    E_TIMEOUT: "KVS_E_TIMEOUT",
    E_TOO_SMALL: "KVS_E_TOO_SMALL",
    E_QUARANTINED: "KVS_E_QUARANTINED",
    E_CLOSED: "KVS_E_CLOSED",
    E_FORMAT: "KVS_E_FORMAT",
}


class KvsError(RuntimeError):
    """A failed C ABI call; `code` is the KVS_E_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class ServerConfig(C.Structure):
    _fields_ = [
        ("device", C.c_int32),
        ("max_keys", C.c_uint32),
        ("unit_bytes", C.c_uint32),
        ("max_key_bytes", C.c_uint32),
        ("heap_bytes", C.c_uint64),
        ("host_pool_bytes", C.c_uint64),
        ("max_value_bytes", C.c_uint64),
        ("shard_id", C.c_uint32),
        ("flags", C.c_uint32),
    ]


class BlockLayout(C.Structure):
    _fields_ = [
        ("n_members", C.c_uint32),
        ("members_per_layer", C.c_uint32),
        ("member_ptrs", C.POINTER(C.c_uint64)),
        ("member_block_bytes", C.POINTER(C.c_uint64)),
        ("n_pool_blocks", C.c_uint64),
    ]


def _u64_struct(name: str, fields: list[str], tail: list[tuple[str, object]] | None = None):
    return type(name, (C.Structure,), {"_fields_": [(f, C.c_uint64) for f in fields] + (tail or [])})


PutProfile = _u64_struct(
    "PutProfile", ["count", "prepare_ns", "program_ns", "enqueue_ns", "landed_wait_ns", "commit_wait_ns", "total_ns"]
)
MoveProfile = _u64_struct(
    "MoveProfile",
    [
        "to_host_count",
        "to_host_worker_ns",
        "to_host_complete_ns",
        "to_host_read_calls",
        "to_host_read_bytes",
        "to_host_read_passes",
        "to_host_read_retries",
        "to_host_read_io_ns",
        "to_host_scatter_ns",
        "to_host_device_pushes",
        "to_device_count",
        "to_device_worker_ns",
        "to_device_complete_ns",
    ],
)
AllocatorProfile = _u64_struct(
    "AllocatorProfile",
    [
        "allocation_calls",
        "allocation_successes",
        "allocation_failures",
        "victim_scans",
        "victims_evicted",
        "lease_calls",
        "lease_successes",
        "lease_failures",
        "lease_victim_scans",
        "lease_victims_evicted",
        "scan_cycles",
        "lease_scan_cycles",
        "allocation_cycles",
    ],
    [("clock_mhz", C.c_uint32)],
)
Stats = _u64_struct(
    "Stats",
    [
        "live_device_bytes",
        "pending_device_bytes",
        "live_keys",
        "device_resident_keys",
        "allocation_calls",
        "allocation_successes",
        "allocation_failures",
        "victims_evicted",
        "catalog_replacements",
        "writes_through",
        "stale_commits",
        "host_serves",
        "admissions",
        "pool_values",
        "heap_values",
    ],
    [("epoch", C.c_uint32), ("issued", C.c_uint32), ("committed", C.c_uint32), ("kernel_launches", C.c_uint64)],
)

class IpcHandle(C.Structure):
    _fields_ = [("bytes", C.c_uint8 * 64)]


class KernelTiming(C.Structure):
    _fields_ = [("launches", C.c_uint64), ("bytes", C.c_uint64), ("total_ms", C.c_double)]


P = C.c_void_p
_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)
_u64p = C.POINTER(C.c_uint64)
_i64p = C.POINTER(C.c_int64)
_intp = C.POINTER(C.c_int)

# name -> (restype, argtypes); every symbol include/kvs.h declares
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kvs_abi_version": (C.c_int, []),
    "kvs_last_error": (C.c_char_p, []),
    "kvs_kernel_launch_count": (C.c_uint64, []),
    "kvs_server_config_default": (C.c_int, [C.POINTER(ServerConfig)]),
    "kvs_server_create": (C.c_int, [C.POINTER(ServerConfig), C.POINTER(P)]),
    "kvs_server_destroy": (C.c_int, [P]),
    "kvs_server_is_ready": (C.c_int, [P, _intp]),
    "kvs_server_moves_completed": (C.c_int, [P, _u64p]),
    "kvs_server_move_profile": (C.c_int, [P, C.POINTER(MoveProfile)]),
    "kvs_server_allocator_profile": (C.c_int, [P, C.POINTER(AllocatorProfile)]),
    "kvs_server_stats": (C.c_int, [P, C.POINTER(Stats)]),
    "kvs_server_device": (C.c_int, [P, _intp]),
    "kvs_server_put_drain_progress": (C.c_int, [P, _u32p, _u32p]),
    "kvs_server_location": (C.c_int, [P, P, C.c_uint32, _intp, _u64p]),
    "kvs_server_index_snapshot": (C.c_int, [P, _u32p, _u32p, C.c_uint32, _u32p]),
    "kvs_server_lru_order": (C.c_int, [P, _u32p, C.c_uint32, _u32p]),
    "kvs_client_create": (C.c_int, [C.POINTER(P), C.c_uint32, C.c_int32, C.POINTER(P)]),
    "kvs_client_destroy": (C.c_int, [P]),
    "kvs_client_is_established": (C.c_int, [P, _intp]),
    "kvs_client_shard_of": (C.c_int, [P, P, C.c_uint32, _u32p]),
    "kvs_ping": (C.c_int, [P, P, C.c_uint32, P, P]),
    "kvs_put": (C.c_int, [P, P, C.c_uint32, P, C.c_uint64, C.c_int, P]),
    "kvs_put_batch": (C.c_int, [P, C.c_uint32, C.POINTER(P), _u32p, C.POINTER(P), _u64p, C.c_int, P]),
    "kvs_get": (C.c_int, [P, P, C.c_uint32, P, C.c_uint64, _intp, _u64p, P]),
    "kvs_get_parallel": (C.c_int, [C.POINTER(P), C.c_uint32, C.POINTER(P), _u32p, P, C.c_uint64, C.c_uint64, _u8p, P]),
    "kvs_exists": (C.c_int, [P, P, C.c_uint32, _intp]),
    "kvs_delete": (C.c_int, [P, P, C.c_uint32, _intp]),
    "kvs_move_to_host": (C.c_int, [P, P, C.c_uint32]),
    "kvs_move_to_device": (C.c_int, [P, P, C.c_uint32]),
    "kvs_flush": (C.c_int, [P]),
    "kvs_client_put_profile": (C.c_int, [P, C.POINTER(PutProfile)]),
    # the block calls take array addresses as plain integers (numpy .ctypes.data): the per-call
    # pointer casts were a measurable part of a one-block get
    "kvs_put_blocks": (C.c_int, [P, C.POINTER(BlockLayout), C.c_uint32, P, P, C.c_int, P]),
    "kvs_get_blocks": (C.c_int, [P, C.POINTER(BlockLayout), C.c_uint32, P, P, P, P]),
    "kvs_exists_batch": (C.c_int, [P, C.c_uint32, P, P]),
    "kvs_restore_chunks": (
        C.c_int,
        [P, C.c_uint32, C.POINTER(P), _u32p, _u32p, C.c_uint32, C.POINTER(P), C.POINTER(P), C.c_uint32, C.c_uint32,
         C.c_uint32, C.POINTER(C.c_int32), C.c_uint32, C.POINTER(C.c_int32), _u8p, P],
    ),
    "kvs_ipc_export": (C.c_int, [P, C.POINTER(IpcHandle), _u64p]),
    "kvs_ipc_open": (C.c_int, [C.c_int32, C.POINTER(IpcHandle), C.POINTER(P)]),
    "kvs_ipc_close": (C.c_int, [C.c_int32, P]),
    "kvs_server_slab": (C.c_int, [P, C.POINTER(P), _u64p]),
    "kvs_serve_gets": (C.c_int, [P, C.c_uint32, C.POINTER(BlockLayout), C.c_uint32, _u32p, _i64p, _u64p, _u8p, P]),
    "kvs_serve_gets_packed": (C.c_int, [P, P, C.c_uint64, C.c_uint32, _u64p, _u8p, P]),
    "kvs_grant_puts": (C.c_int, [P, C.c_uint32, _u64p, C.c_uint64, _u64p, _u32p]),
    "kvs_puts_landed": (C.c_int, [P, P]),
    "kvs_copy_blocks": (C.c_int, [P, C.POINTER(BlockLayout), C.c_uint32, _i64p, _u64p, C.c_int, P]),
    "kvs_copy_values": (C.c_int, [P, P, C.c_uint64, C.c_uint32, _u64p, C.c_int, P]),
    "kvs_paged_fill_varlen": (
        C.c_int,
        [P, P, C.c_uint32, C.c_uint32, C.c_uint32, P, C.c_uint32, P, C.c_uint32, P, P, P, C.c_uint32, C.c_uint32, P, P],
    ),
    "kvs_paged_fill_varlen_layers": (
        C.c_int,
        [C.c_uint32, C.POINTER(P), C.POINTER(P), C.c_uint32, C.c_uint32, C.c_uint32, P, C.c_uint32, P, C.c_uint32, P,
         C.POINTER(P), C.POINTER(P), C.c_uint32, C.c_uint32, P, P],
    ),
    "kvs_client_set_timing": (C.c_int, [P, C.c_int]),
    "kvs_client_timing": (C.c_int, [P, C.POINTER(KernelTiming), C.POINTER(KernelTiming)]),
    "kvs_client_host_tier_timing": (C.c_int, [P, C.POINTER(KernelTiming), C.POINTER(KernelTiming)]),
    "kvs_server_set_timing": (C.c_int, [P, C.c_int]),
    "kvs_server_write_through_timing": (C.c_int, [P, C.POINTER(KernelTiming)]),
    "kvs_gather_chunk": (
        C.c_int,
        [_u64p, C.c_uint32, C.c_uint32, _u64p, _u64p, _u32p, C.c_uint32, _u64p, _u32p, C.c_uint32, P, C.c_uint64, P],
    ),
    "kvs_gather_chunk_noalloc": (
        C.c_int,
        [_u64p, C.c_uint32, C.c_uint32, _u64p, _u64p, _u32p, C.c_uint32, _u64p, _u32p, C.c_uint32, P, C.c_uint64, P],
    ),
    "kvs_scatter_chunk": (
        C.c_int,
        [P, C.c_uint64, _u64p, C.c_uint32, C.c_uint32, _u64p, _u64p, _u32p, C.c_uint32, _u64p, P],
    ),
    "kvs_copy_engine_status": (C.c_int, [C.c_int32, _u32p, _u32p]),
    "kvs_set_copy_wait_limit": (C.c_int, [C.c_int64]),
    "kvs_set_small_copy_limit": (C.c_int, [C.c_int64]),
    "kvs_bucket_requests": (C.c_int, [C.c_int32, P, P, C.c_uint32, C.c_uint32, P, C.c_uint32, C.c_uint32, C.c_int64,
                                      P, P, P, P, P]),
}

_lib = None


def load(path: str | os.PathLike | None = None):
    """Load (once) and return the product library with every signature declared."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    target = Path(path) if path else LIB_PATH
    if not target.exists():
        raise ImportError(
            f"kvcache-manager requires its native extension {target.name}; build it with "
            f"`python tt-infinity_b200/build.py` (or __graft_entry__.build())"
        )
    lib = C.CDLL(str(target), mode=C.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.kvs_abi_version() != KVS_ABI_VERSION:
        raise ImportError(
            f"kvcache-manager requires KV store C ABI {KVS_ABI_VERSION}, but loaded ABI {lib.kvs_abi_version()}"
        )
    if path is None:
        _lib = lib
        _bind_fastcall(lib)
    return lib


fastcall = None  # the CPython module of the block calls' hot path, bound to the loaded library


def _bind_fastcall(lib) -> None:
    """Hands the loaded library's block-call entry points to the _fastcall module (built beside the
    library by build.py). Without it the facade calls the same entry points through ctypes."""
    global fastcall
    try:
        from . import _fastcall
    except ImportError:
        return
    addr = lambda fn: C.cast(fn, C.c_void_p).value
    _fastcall.bind(addr(lib.kvs_put_blocks), addr(lib.kvs_get_blocks), addr(lib.kvs_exists_batch))
    fastcall = _fastcall


def check(rc: int) -> None:
    if rc != OK:
        msg = load().kvs_last_error().decode(errors="replace")
        raise KvsError(rc, f"{msg} [{_ERROR_NAMES.get(rc, rc)}]")


def struct_to_dict(s) -> dict:
    return {name: getattr(s, name) for name, _ in s._fields_}
