"""The C ABI library loads on CPU and exports exactly what include/kvs.h declares.

No compute call runs here (there is no GPU): only symbol presence, the ABI version, the
environment-knob parsing of kvs_server_config_default, and argument validation that fails before
touching a device.
"""

import ctypes as C
import os
import re
from pathlib import Path

import pytest

from kvcache_manager import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "kvs.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(kvs_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    return _native.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = declared_functions()
    assert len(names) >= 35
    raw = C.CDLL(str(_native.LIB_PATH))
    for n in names:
        assert hasattr(raw, n), f"{n} declared in kvs.h but not exported"
    assert set(names) == set(_native.SIGNATURES), set(names) ^ set(_native.SIGNATURES)


def test_abi_version(lib):
    assert lib.kvs_abi_version() == _native.KVS_ABI_VERSION == 1


def test_config_defaults_restate_reference_defaults(lib, monkeypatch):
    for k in ("KVM_SERVER_DRAM_MAX_KEYS", "KVM_SERVER_DRAM_VALUE_HEAP_BYTES", "KVM_SERVER_HOST_POOL_BYTES",
              "KVM_COMMON_MAX_VALUE_BYTES", "KVM_SERVER_MAX_KEY_BYTES"):
        monkeypatch.delenv(k, raising=False)
    cfg = _native.ServerConfig()
    assert lib.kvs_server_config_default(C.byref(cfg)) == 0
    assert cfg.max_keys == 1024  # kMaxKeysDefault
    assert cfg.heap_bytes == 1_434_541_824  # kValueHeapBytesDefault
    assert cfg.unit_bytes == 4288  # kMaxChunkValueBytes
    assert cfg.max_key_bytes == 128  # kMaxPutKeyBytes
    assert cfg.max_value_bytes == 64 << 20  # kMaxMultiChunkValueBytesDefault


@pytest.mark.parametrize("bad", ["", " 1", "1 ", "+1", "-1", "1x", "18446744073709551616"])
def test_config_env_parsing_is_exact(lib, monkeypatch, bad):
    monkeypatch.setenv("KVM_SERVER_DRAM_MAX_KEYS", bad)
    cfg = _native.ServerConfig()
    assert lib.kvs_server_config_default(C.byref(cfg)) == _native.E_INVAL
    assert b"KVM_SERVER_DRAM_MAX_KEYS" in lib.kvs_last_error()


def test_config_env_overrides(lib, monkeypatch):
    monkeypatch.setenv("KVM_SERVER_DRAM_MAX_KEYS", "1048576")
    monkeypatch.setenv("KVM_SERVER_MAX_KEY_BYTES", "64")
    cfg = _native.ServerConfig()
    assert lib.kvs_server_config_default(C.byref(cfg)) == 0
    assert cfg.max_keys == 1 << 20 and cfg.max_key_bytes == 64
    monkeypatch.setenv("KVM_SERVER_MAX_KEY_BYTES", "129")
    assert lib.kvs_server_config_default(C.byref(cfg)) == _native.E_INVAL


def test_null_and_invalid_arguments_fail_without_a_device(lib):
    h = C.c_void_p()
    assert lib.kvs_server_create(None, C.byref(h)) == _native.E_INVAL
    assert lib.kvs_client_create(None, 0, 0, C.byref(h)) == _native.E_INVAL
    assert lib.kvs_server_destroy(None) == 0
    assert lib.kvs_client_destroy(None) == 0
    found = C.c_int()
    assert lib.kvs_exists(None, b"k", 1, C.byref(found)) == _native.E_INVAL
    # chunk op validation runs before any device access
    ptrs = (C.c_uint64 * 1)(1)
    sbb = (C.c_uint64 * 1)(30)  # not 4-byte aligned
    ext = (C.c_uint64 * 1)(1 << 20)
    ids = (C.c_uint32 * 1)(0)
    rb = (C.c_uint64 * 1)(32)
    assert lib.kvs_gather_chunk(ptrs, 1, 1, sbb, ext, ids, 1, rb, None, 0, C.c_void_p(1), 1 << 20, None) == _native.E_INVAL
    assert b"4-byte aligned" in lib.kvs_last_error()
    sbb[0] = 32
    hw = (C.c_uint32 * 4)(1, 2, 3, 4)  # 16-byte header
    assert lib.kvs_gather_chunk(ptrs, 1, 1, sbb, ext, ids, 1, rb, hw, 4, C.c_void_p(1), 1 << 20, None) == _native.E_INVAL
    assert b"header must be 32-byte aligned" in lib.kvs_last_error()


def test_more_entry_points_validate_before_any_device_access(lib):
    P = C.c_void_p
    arr = (P * 1)(P(1))
    # paged fill: nothing to do for zero layers, then argument checks in the reference's order
    assert lib.kvs_paged_fill_varlen_layers(0, None, None, 1, 32, 64, None, 1, None, 1, None, None, None, 4, 16,
                                            None, None) == 0
    assert lib.kvs_paged_fill_varlen_layers(1, None, arr, 1, 32, 64, None, 1, None, 1, None, arr, arr, 4, 16,
                                            None, None) == _native.E_INVAL
    assert b"layer arrays are null" in lib.kvs_last_error()
    assert lib.kvs_paged_fill_varlen_layers(1, arr, arr, 1, 32, 64, None, 0, None, 1, None, arr, arr, 4, 16,
                                            None, None) == _native.E_INVAL
    assert b"at least one row" in lib.kvs_last_error()
    assert lib.kvs_paged_fill_varlen(P(1), P(1), 1, 32, 64, None, 1, None, 8, None, P(1), P(1), 4, 16, None,
                                     None) == _native.E_INVAL
    assert b"must be <= max_num_blocks" in lib.kvs_last_error()
    assert lib.kvs_paged_fill_varlen(P(1), P(1), 1, 32, 64, None, 1, None, 1, None, P(1), P(1), 4, 0, None,
                                     None) == _native.E_INVAL
    assert b"must be > 0" in lib.kvs_last_error()
    # batch limits and null handles
    assert lib.kvs_put_batch(None, 129, None, None, None, None, 0, None) == _native.E_INVAL
    assert b"128-descriptor limit" in lib.kvs_last_error()
    found = (C.c_uint8 * 1)()
    assert lib.kvs_get_parallel(None, 0, None, None, P(1), 0, 1, found, None) == _native.E_INVAL
    h = _native.IpcHandle()
    off = C.c_uint64()
    assert lib.kvs_ipc_export(None, C.byref(h), C.byref(off)) == _native.E_INVAL
    assert lib.kvs_ipc_open(0, None, None) == _native.E_INVAL


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError, match="requires its native extension"):
        _native.load(tmp_path / "libkvs_b200.so")


def test_oracle_is_not_importable_from_the_product():
    pkg = Path(__file__).resolve().parents[1] / "tt-infinity_b200"
    for p in pkg.rglob("*"):
        if p.suffix in (".py", ".cu", ".cuh", ".cpp", ".hpp", ".h"):
            assert "oracle" not in p.read_text().replace("oracles", ""), p
    assert os.path.exists(_native.LIB_PATH)


def test_new_entry_points_check_their_arguments_without_a_device(lib):
    # the chunk restore needs a client; a null handle fails before anything else
    assert lib.kvs_restore_chunks(None, 1, None, None, None, 1, None, None, 8, 16, 256, None, 1, None, None,
                                  None) == _native.E_INVAL
    assert b"client handle is null" in lib.kvs_last_error()
    # copy-engine health: null outputs are refused, and the wait limit takes at most 2^32 - 1 polls
    unsafe = C.c_uint32()
    assert lib.kvs_copy_engine_status(0, None, C.byref(unsafe)) == _native.E_INVAL
    assert lib.kvs_set_copy_wait_limit(1 << 33) == _native.E_INVAL
    assert b"2^32 - 1" in lib.kvs_last_error()
    assert lib.kvs_set_copy_wait_limit(-1) == 0  # the default
    # timing calls need their handles
    t = _native.KernelTiming()
    assert lib.kvs_server_set_timing(None, 1) == _native.E_INVAL
    assert lib.kvs_server_write_through_timing(None, C.byref(t)) == _native.E_INVAL
    assert lib.kvs_client_host_tier_timing(None, C.byref(t), C.byref(t)) == _native.E_INVAL


def test_fastcall_module_is_bound_and_takes_only_exact_arrays(lib):
    """The CPython module of the block calls is built beside the library and bound to it. It calls
    the C ABI only with 1-D uint64 keys and int64 block ids of equal length (else NotImplemented,
    and the facade converts); a failing call comes back as the library's error code."""
    import numpy as np

    fast = _native.fastcall
    assert fast is not None, "the _fastcall module was not built or not bound"
    keys, ids = np.arange(3, dtype=np.uint64), np.arange(3, dtype=np.int64)
    assert fast.get_blocks(0, 0, keys, ids, 0) == _native.E_INVAL  # null client: checked before any device work
    assert "client handle is null" in lib.kvs_last_error().decode()
    assert fast.put_blocks(0, 0, keys, ids, False, 0) == _native.E_INVAL
    assert fast.exists_batch(0, keys) == _native.E_INVAL
    assert fast.get_blocks(0, 0, keys.astype(np.int64), ids, 0) is NotImplemented
    assert fast.get_blocks(0, 0, keys, ids.astype(np.int32), 0) is NotImplemented
    assert fast.get_blocks(0, 0, keys, ids[:2], 0) is NotImplemented
    assert fast.get_blocks(0, 0, [1, 2, 3], ids, 0) is NotImplemented
    assert fast.get_blocks(0, 0, keys[::2], ids[:2], 0) is NotImplemented  # not contiguous
    assert fast.exists_batch(0, keys.reshape(1, 3)) is NotImplemented


def test_bucket_requests_argument_checks_before_any_device_work(lib):
    """kvs_bucket_requests refuses a bad shard count, capacity, get count or a missing array before
    it touches a device."""
    buf = C.create_string_buffer(64)
    p = C.cast(buf, C.c_void_p)
    cases = [
        (0, 8, 0, 0, "world 0 outside"),
        (33, 8, 0, 0, "world 33 outside"),
        (2, 0, 0, 0, "cap must be positive"),
        (2, 8, 1, 2, "2 gets of 1 keys"),
    ]
    for world, cap, n, n_get, msg in cases:
        rc = lib.kvs_bucket_requests(0, p, p, n, n_get, None, world, cap, 0, p, p, p, p, None)
        assert rc == _native.E_INVAL and msg in lib.kvs_last_error().decode(), (world, cap, n, n_get)
    assert lib.kvs_bucket_requests(0, None, None, 3, 0, None, 2, 8, 0, p, p, p, p, None) == _native.E_INVAL
    assert "null argument" in lib.kvs_last_error().decode()
    assert lib.kvs_bucket_requests(0, p, p, 1, 0, None, 2, 8, 0, p, p, p, None, None) == _native.E_INVAL
    # host memory is refused (device memory of the named GPU only)
    assert lib.kvs_bucket_requests(0, p, p, 1, 0, None, 2, 8, 0, p, p, p, p, None) == _native.E_INVAL
    assert "device memory" in lib.kvs_last_error().decode()
