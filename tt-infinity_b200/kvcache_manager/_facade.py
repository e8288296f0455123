"""Product facades: `Server` (one store shard on one B200) and `Client`.

Method names, argument meaning and error behaviour follow the reference's
src/kvcache_manager/_facade.py:34-170 and include/kvcache_manager/client.hpp:26-66 /
server.hpp:21-55. The device handle is a CUDA device ordinal (or torch.device) instead of a TT
mesh, tensors are torch CUDA tensors instead of TTNN DRAM tensors, and the Fabric routing
arguments (server_node, client_coord, static inter-mesh lanes) are replaced by the list of shards
a client addresses. The paged-block calls put_blocks / get_blocks / exists_batch are the B200
main path: one gather / scatter kernel moves a whole batch of paged KV blocks.
"""

from __future__ import annotations

import ctypes as C
from types import TracebackType
from typing import Any, Iterable, Sequence

import numpy as np

from . import _native
from ._native import KvsError, check, load, struct_to_dict


def _torch():
    import torch

    return torch


def to_key(value: Any) -> bytes:
    """Normalise a key: str (utf-8), bytes, or a 64-bit integer (8 little-endian bytes).

    Mirrors the nanobind `to_key` of src/python/bindings.cpp:77-86, plus the 64-bit chained
    prefix-hash keys of the paged-block path."""
    if isinstance(value, str):
        return value.encode("utf-8")
    if isinstance(value, (bytes, bytearray, memoryview)):
        return bytes(value)
    if isinstance(value, (int, np.integer)):
        v = int(value)
        if not 0 <= v < (1 << 64):
            raise ValueError("integer keys must be unsigned 64-bit values")
        return v.to_bytes(8, "little")
    raise TypeError("key must be str or bytes")


def _device_index(device: Any) -> int:
    if isinstance(device, int):
        return device
    torch = _torch()
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError(f"device must be a CUDA device, got {d}")
    return 0 if d.index is None else d.index


_raw_stream = None


def _stream_handle(device: int) -> int:
    """The caller's current CUDA stream on `device` as a raw handle."""
    global _raw_stream
    if _raw_stream is None:
        torch = _torch()
        _raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None) or (
            lambda d: torch.cuda.current_stream(d).cuda_stream)
    return _raw_stream(device)


def _check_tensor(t: Any, device: int, op: str) -> None:
    torch = _torch()
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{op}: tensor must be a torch.Tensor")
    if t.device.type != "cuda":
        raise RuntimeError(f"{op}: tensor must use DEVICE storage")
    if t.device.index != device:
        raise RuntimeError(f"{op}: tensor must belong to the client device {device}; got device {t.device.index}")
    if not t.is_contiguous():
        raise RuntimeError(f"{op}: tensor must be contiguous")


class Server:
    """Own one KV store shard: device slab + index replica on `device`, pinned host tier."""

    def __init__(
        self,
        device: Any = 0,
        *,
        max_keys: int | None = None,
        heap_bytes: int | None = None,
        host_pool_bytes: int | None = None,
        max_key_bytes: int | None = None,
        max_value_bytes: int | None = None,
        unit_bytes: int | None = None,
        worker_group: int = 0,
        profile: bool = False,
    ) -> None:
        lib = load()
        cfg = _native.ServerConfig()
        check(lib.kvs_server_config_default(C.byref(cfg)))
        cfg.device = _device_index(device)
        if max_keys is not None:
            cfg.max_keys = max_keys
        if heap_bytes is not None:
            cfg.heap_bytes = heap_bytes
        if host_pool_bytes is not None:
            cfg.host_pool_bytes = host_pool_bytes
        if max_key_bytes is not None:
            cfg.max_key_bytes = max_key_bytes
        if max_value_bytes is not None:
            cfg.max_value_bytes = max_value_bytes
        if unit_bytes is not None:
            cfg.unit_bytes = unit_bytes
        cfg.shard_id = worker_group
        cfg.flags = 1 if profile else 0
        handle = C.c_void_p()
        check(lib.kvs_server_create(C.byref(cfg), C.byref(handle)))
        self._h = handle
        self.config = {n: getattr(cfg, n) for n, _ in cfg._fields_}

    @property
    def device(self) -> int:
        return self.config["device"]

    def _handle(self) -> C.c_void_p:
        if not self._h:
            raise KvsError(_native.E_CLOSED, "server is closed")
        return self._h

    def is_ready(self) -> bool:
        if not self._h:
            return False
        v = C.c_int()
        check(load().kvs_server_is_ready(self._h, C.byref(v)))
        return bool(v.value)

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, None
            check(load().kvs_server_destroy(h))

    def moves_completed(self) -> int:
        v = C.c_uint64()
        check(load().kvs_server_moves_completed(self._handle(), C.byref(v)))
        return v.value

    def move_profile(self) -> dict[str, Any]:
        p = _native.MoveProfile()
        check(load().kvs_server_move_profile(self._handle(), C.byref(p)))
        return struct_to_dict(p)

    def allocator_profile(self) -> dict[str, Any]:
        p = _native.AllocatorProfile()
        check(load().kvs_server_allocator_profile(self._handle(), C.byref(p)))
        return struct_to_dict(p)

    def stats(self) -> dict[str, Any]:
        p = _native.Stats()
        check(load().kvs_server_stats(self._handle(), C.byref(p)))
        return struct_to_dict(p)

    def location(self, key: Any) -> tuple[int, int]:
        k = to_key(key)
        loc, off = C.c_int(), C.c_uint64()
        check(load().kvs_server_location(self._handle(), k, len(k), C.byref(loc), C.byref(off)))
        return loc.value, off.value

    def lru_order(self) -> list[int]:
        n = C.c_uint32()
        check(load().kvs_server_lru_order(self._handle(), None, 0, C.byref(n)))
        buf = (C.c_uint32 * max(1, n.value))()
        check(load().kvs_server_lru_order(self._handle(), buf, n.value, C.byref(n)))
        return list(buf[: n.value])

    def index_snapshot(self) -> tuple[np.ndarray, np.ndarray]:
        """(host, device) hash buckets as ({hash, slot} pairs) arrays of shape (n_buckets, 2)."""
        nb = C.c_uint32()
        check(load().kvs_server_index_snapshot(self._handle(), None, None, 0, C.byref(nb)))
        host = np.zeros((nb.value, 2), np.uint32)
        dev = np.zeros((nb.value, 2), np.uint32)
        check(
            load().kvs_server_index_snapshot(
                self._handle(),
                host.ctypes.data_as(_native._u32p),
                dev.ctypes.data_as(_native._u32p),
                nb.value,
                C.byref(nb),
            )
        )
        return host, dev

    def set_write_through_timing(self, enable: bool) -> None:
        """Bracket every batch of write-through copies with CUDA events on the write-through stream."""
        check(load().kvs_server_set_timing(self._handle(), 1 if enable else 0))

    def write_through_timing(self) -> dict[str, float]:
        """Totals since the last call: batches ("launches"), bytes copied to the host tier and their
        device time (total_ms)."""
        t = _native.KernelTiming()
        check(load().kvs_server_write_through_timing(self._handle(), C.byref(t)))
        return struct_to_dict(t)

    def _test_put_drain_progress(self) -> tuple[int, int]:
        i, c = C.c_uint32(), C.c_uint32()
        check(load().kvs_server_put_drain_progress(self._handle(), C.byref(i), C.byref(c)))
        return i.value, c.value

    def __enter__(self) -> "Server":
        return self

    def __exit__(
        self,
        exc_type: type[BaseException] | None,
        exc_value: BaseException | None,
        traceback: TracebackType | None,
    ) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class PagedLayout:
    """A paged KV cache as the block calls see it: per layer K, V (and optional extra members,
    e.g. per-block scales), each a CUDA tensor whose first dimension is the block index.

    Built from vLLM-style caches with `PagedLayout.from_kv_caches([(k0, v0), (k1, v1), ...])`
    where every tensor is (num_blocks, kv_heads, block_size, head_dim) -- the reference's TT
    layout per layer (patch 0005 lines 10713-10760)."""

    def __init__(self, members: Sequence[Any], members_per_layer: int = 2) -> None:
        torch = _torch()
        if not members:
            raise ValueError("layout: members must not be empty")
        if len(members) % members_per_layer:
            raise ValueError("layout: members must be whole layers")
        dev = members[0].device
        nblocks = members[0].shape[0]
        bb = []
        for i, t in enumerate(members):
            if not isinstance(t, torch.Tensor) or t.device != dev:
                raise ValueError(f"layout: member {i} must be a tensor on {dev}")
            if not t.is_contiguous():
                raise ValueError(f"layout: member {i} must be contiguous")
            if t.shape[0] != nblocks:
                raise ValueError(f"layout: member {i} has {t.shape[0]} blocks, member 0 has {nblocks}")
            bb.append(t.numel() * t.element_size() // nblocks)
        self.members = list(members)
        self.members_per_layer = members_per_layer
        self.num_blocks = int(nblocks)
        self.device = dev.index if dev.index is not None else 0
        self.member_block_bytes = bb
        self._ptrs = (C.c_uint64 * len(members))(*[t.data_ptr() for t in members])
        self._bytes = (C.c_uint64 * len(members))(*bb)
        self.c = _native.BlockLayout(len(members), members_per_layer, self._ptrs, self._bytes, self.num_blocks)
        self.ref = C.byref(self.c)  # reused by every call
        self.addr = C.addressof(self.c)  # the same, as an integer for the _fastcall module

    @classmethod
    def from_kv_caches(cls, kv_caches: Iterable[Sequence[Any]]) -> "PagedLayout":
        members: list[Any] = []
        per = None
        for layer in kv_caches:
            layer = list(layer)
            if per is None:
                per = len(layer)
            elif per != len(layer):
                raise ValueError("layout: every layer must have the same members")
            members += layer
        return cls(members, per or 2)

    @property
    def n_layers(self) -> int:
        return len(self.members) // self.members_per_layer

    def value_bytes(self) -> int:
        """Byte length of one block's stored value (header + every member's block)."""
        hdr = 4 * (2 + self.n_layers)
        hdr = (hdr + 31) // 32 * 32
        off = hdr
        for b in self.member_block_bytes:
            off = (off + b + 15) // 16 * 16
        return off


def _i64_array(values: Any) -> np.ndarray:
    if isinstance(values, np.ndarray) and values.dtype == np.int64 and values.flags.c_contiguous:
        return values
    return np.ascontiguousarray(np.asarray(values, dtype=np.int64))


def _addr(a: np.ndarray) -> int:
    """Address of a C-contiguous array's first element: through the buffer protocol when the
    array is writable (a third of the cost of `ndarray.ctypes`), else `ndarray.ctypes`."""
    try:
        return C.addressof(C.c_char.from_buffer(a))
    except (TypeError, ValueError):  # read-only or empty
        return a.ctypes.data


def _u64_keys(keys: Any) -> np.ndarray:
    if isinstance(keys, np.ndarray) and keys.dtype == np.uint64 and keys.flags.c_contiguous:
        return keys
    arr = np.asarray(keys)
    if arr.dtype.kind in "iu":
        return np.ascontiguousarray(arr.astype(np.uint64))
    return np.ascontiguousarray(np.array([int.from_bytes(to_key(k)[:8].ljust(8, b"\0"), "little") for k in keys], np.uint64))


class Client:
    """A KV store client on one GPU; keys are hash-sharded over `server` (one or many shards)."""

    def __init__(self, device: Any = 0, server: Server | Sequence[Server] | None = None) -> None:
        if server is None:
            raise ValueError("a Client requires server (a Server or a list of shard Servers)")
        shards = [server] if isinstance(server, Server) else list(server)
        if not shards:
            raise ValueError("a Client requires at least one server shard")
        self.device = _device_index(device)
        self._servers = shards  # keep the shards alive while the client lives
        arr = (C.c_void_p * len(shards))(*[s._handle().value for s in shards])
        handle = C.c_void_p()
        check(load().kvs_client_create(arr, len(shards), self.device, C.byref(handle)))
        self._h = handle
        self._hv = handle.value  # the handle as an integer for the _fastcall module; 0 once closed

    def _handle(self) -> C.c_void_p:
        if not self._h:
            raise KvsError(_native.E_CLOSED, "client is closed")
        return self._h

    def is_established(self) -> bool:
        if not self._h:
            return False
        v = C.c_int()
        check(load().kvs_client_is_established(self._h, C.byref(v)))
        return bool(v.value)

    def close(self) -> None:
        if self._h:
            h, self._h, self._hv = self._h, None, 0
            check(load().kvs_client_destroy(h))

    def shard_of(self, key: Any) -> int:
        k = to_key(key)
        v = C.c_uint32()
        check(load().kvs_client_shard_of(self._handle(), k, len(k), C.byref(v)))
        return v.value

    def ping(self, payload: bytes) -> bytes:
        payload = bytes(payload)
        out = C.create_string_buffer(max(1, len(payload)))
        check(load().kvs_ping(self._handle(), payload, len(payload), out, _stream_handle(self.device)))
        return out.raw[: len(payload)]

    def put(self, key: Any, value_tensor: Any, value_len_bytes: int, sync_commit: bool = False) -> None:
        k = to_key(key)
        _check_tensor(value_tensor, self.device, "put")
        nbytes = value_tensor.numel() * value_tensor.element_size()
        if value_len_bytes > nbytes:
            raise RuntimeError(f"put: value_len {value_len_bytes} exceeds tensor packed bytes {nbytes}")
        check(
            load().kvs_put(
                self._handle(), k, len(k), C.c_void_p(value_tensor.data_ptr()), value_len_bytes,
                1 if sync_commit else 0, _stream_handle(self.device),
            )
        )

    def put_batch(
        self, keys: list[Any], value_tensors: list[Any], value_len_bytes: list[int], sync_commit: bool = False
    ) -> None:
        if not (len(keys) == len(value_tensors) == len(value_len_bytes)):
            raise RuntimeError("put_batch: keys, value_tensors and value_len_bytes must have equal length")
        ks = [to_key(k) for k in keys]
        for t, n in zip(value_tensors, value_len_bytes):
            _check_tensor(t, self.device, "put_batch")
            if n > t.numel() * t.element_size():
                raise RuntimeError(f"put_batch: value_len {n} exceeds tensor packed bytes")
        kbufs = [C.create_string_buffer(k, len(k)) for k in ks]
        karr = (C.c_void_p * len(ks))(*[C.addressof(b) for b in kbufs])
        klen = (C.c_uint32 * len(ks))(*[len(k) for k in ks])
        varr = (C.c_void_p * len(ks))(*[t.data_ptr() for t in value_tensors])
        vlen = (C.c_uint64 * len(ks))(*value_len_bytes)
        check(
            load().kvs_put_batch(
                self._handle(), len(ks), karr, klen, varr, vlen, 1 if sync_commit else 0, _stream_handle(self.device)
            )
        )

    def put_profile(self) -> dict[str, Any]:
        p = _native.PutProfile()
        check(load().kvs_client_put_profile(self._handle(), C.byref(p)))
        return struct_to_dict(p)

    def flush(self) -> None:
        check(load().kvs_flush(self._handle()))

    def get(self, key: Any, out_tensor: Any) -> bool:
        k = to_key(key)
        _check_tensor(out_tensor, self.device, "get")
        cap = out_tensor.numel() * out_tensor.element_size()
        if cap == 0:
            raise RuntimeError("get: out_tensor packed byte size must be > 0")
        found, vlen = C.c_int(), C.c_uint64()
        check(
            load().kvs_get(
                self._handle(), k, len(k), C.c_void_p(out_tensor.data_ptr()), cap, C.byref(found), C.byref(vlen),
                _stream_handle(self.device),
            )
        )
        return bool(found.value)

    @staticmethod
    def get_parallel(clients: list["Client"], keys: list[Any], out_tensor: Any) -> list[bool]:
        """clients[i] reads keys[i] into row i of out_tensor (rows of equal byte size)."""
        if not clients:
            raise RuntimeError("get_parallel: clients must not be empty")
        if len(clients) != len(keys):
            raise RuntimeError(
                f"get_parallel: clients and keys must have equal length ({len(clients)} != {len(keys)})"
            )
        dev = clients[0].device
        _check_tensor(out_tensor, dev, "get_parallel")
        total = out_tensor.numel() * out_tensor.element_size()
        stride = total // len(clients)
        ks = [to_key(k) for k in keys]
        kbufs = [C.create_string_buffer(k, len(k)) for k in ks]
        carr = (C.c_void_p * len(clients))(*[c._handle().value for c in clients])
        karr = (C.c_void_p * len(ks))(*[C.addressof(b) for b in kbufs])
        klen = (C.c_uint32 * len(ks))(*[len(k) for k in ks])
        found = (C.c_uint8 * len(ks))()
        check(
            load().kvs_get_parallel(
                carr, len(clients), karr, klen, C.c_void_p(out_tensor.data_ptr()), stride, stride, found,
                _stream_handle(dev),
            )
        )
        return [bool(f) for f in found]

    def exists(self, key: Any) -> bool:
        k = to_key(key)
        f = C.c_int()
        check(load().kvs_exists(self._handle(), k, len(k), C.byref(f)))
        return bool(f.value)

    def delete(self, key: Any) -> bool:
        k = to_key(key)
        f = C.c_int()
        check(load().kvs_delete(self._handle(), k, len(k), C.byref(f)))
        return bool(f.value)

    remove = delete

    def move_to_host(self, key: Any) -> None:
        k = to_key(key)
        check(load().kvs_move_to_host(self._handle(), k, len(k)))

    def move_to_device(self, key: Any) -> None:
        k = to_key(key)
        check(load().kvs_move_to_device(self._handle(), k, len(k)))

    # ---- paged-block path
    def put_blocks(self, layout: PagedLayout, keys: Any, block_ids: Any, sync_commit: bool = False) -> None:
        if layout.device != self.device:
            raise RuntimeError(f"put_blocks: layout lives on device {layout.device}, client on {self.device}")
        fast = _native.fastcall
        if fast is not None and self._hv:  # uint64 / int64 arrays of equal length go straight to the C ABI
            rc = fast.put_blocks(self._hv, layout.addr, keys, block_ids, sync_commit, _stream_handle(self.device))
            if rc is not NotImplemented:
                check(rc)
                return
        k = _u64_keys(keys)
        b = _i64_array(block_ids)
        if k.shape != b.shape:
            raise RuntimeError("put_blocks: keys and block_ids must have equal length")
        check(load().kvs_put_blocks(self._handle(), layout.ref, k.size, _addr(k), _addr(b),
                                    1 if sync_commit else 0, _stream_handle(self.device)))

    def get_blocks(self, layout: PagedLayout, keys: Any, block_ids: Any) -> np.ndarray:
        if layout.device != self.device:
            raise RuntimeError(f"get_blocks: layout lives on device {layout.device}, client on {self.device}")
        fast = _native.fastcall
        if fast is not None and self._hv:  # uint64 / int64 arrays of equal length go straight to the C ABI
            r = fast.get_blocks(self._hv, layout.addr, keys, block_ids, _stream_handle(self.device))
            if r.__class__ is np.ndarray:
                return r
            if r is not NotImplemented:
                check(r)
        k = _u64_keys(keys)
        b = _i64_array(block_ids)
        if k.shape != b.shape:
            raise RuntimeError("get_blocks: keys and block_ids must have equal length")
        found = np.zeros(k.size, np.bool_)  # bool is one byte: the C ABI fills it in place
        check(load().kvs_get_blocks(self._handle(), layout.ref, k.size, _addr(k), _addr(b), _addr(found),
                                    _stream_handle(self.device)))
        return found

    def exists_batch(self, keys: Any) -> np.ndarray:
        fast = _native.fastcall
        if fast is not None and self._hv:
            r = fast.exists_batch(self._hv, keys)
            if r.__class__ is np.ndarray:
                return r
            if r is not NotImplemented:
                check(r)
        k = _u64_keys(keys)
        found = np.zeros(k.size, np.bool_)
        check(load().kvs_exists_batch(self._handle(), k.size, _addr(k), _addr(found)))
        return found

    def set_kernel_timing(self, enable: bool) -> None:
        """Bracket every gather / scatter launch with CUDA events on the client stream."""
        check(load().kvs_client_set_timing(self._handle(), 1 if enable else 0))

    def kernel_timing(self) -> dict[str, dict[str, float]]:
        """Totals since the last call: {"gather": {...}, "scatter": {...}} (launches, bytes, total_ms)."""
        g, s = _native.KernelTiming(), _native.KernelTiming()
        check(load().kvs_client_timing(self._handle(), C.byref(g), C.byref(s)))
        return {"gather": struct_to_dict(g), "scatter": struct_to_dict(s)}

    def host_tier_timing(self) -> dict[str, dict[str, float]]:
        """Totals since the last call of the host-tier copy launches of gets (timing on):
        {"admissions": {...}, "serves": {...}} (launches, bytes, total_ms)."""
        a, s = _native.KernelTiming(), _native.KernelTiming()
        check(load().kvs_client_host_tier_timing(self._handle(), C.byref(a), C.byref(s)))
        return {"admissions": struct_to_dict(a), "serves": struct_to_dict(s)}

    def __enter__(self) -> "Client":
        return self

    def __exit__(
        self,
        exc_type: type[BaseException] | None,
        exc_value: BaseException | None,
        traceback: TracebackType | None,
    ) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
