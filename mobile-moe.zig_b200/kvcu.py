"""Python binding of libkvcuda.so (include/kvcuda.h) over ctypes.

This is the Python-side mirror of mobile-moe.zig's KV-cache interface
(src/kv_cache.zig) for users and tests: `KVCache` keeps the reference's
method names (ensureCapacity, put, getKVCompressed, getKPe, saveToFile, ...)
and raises `KVCudaError` where the Zig code returns an error (the `.name`
attribute is the reference's error name, e.g. "OutOfKVCacheBlocks").

Every data operation runs on the GPU through the C-ABI; there is no CPU
fallback.  If libkvcuda.so has not been built, importing works but the first
call raises with instructions (python mobile-moe.zig_b200/build.py).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkvcuda.so")

ERROR_NAMES = {
    -1: "OutOfKVCacheBlocks", -2: "PositionOutOfBounds", -3: "LayerOutOfBounds",
    -4: "PositionNotWritten", -5: "PrefixCacheMiss", -6: "InvalidCheckpointMagic",
    -7: "UnsupportedCheckpointVersion", -8: "CheckpointShapeMismatch", -9: "EndOfStream",
    -10: "IoError", -11: "InvalidArgument", -12: "CudaError", -13: "DeviceStatus",
    -14: "OutOfMemory", -15: "BadBlockId", -16: "Unsupported", -17: "NoDevice",
}
NO_HASH = (1 << 64) - 1
DECODE_AUTO, DECODE_CUDA_CORE, DECODE_TENSOR_CORE = 0, 1, 2


class KVCudaError(RuntimeError):
    def __init__(self, code: int, what: str, detail: str):
        self.code = code
        self.name = ERROR_NAMES.get(code, f"error{code}")
        super().__init__(f"{what}: {self.name} ({code}): {detail}")


class PoolDesc(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("num_blocks", C.c_uint32), ("block_size", C.c_uint32),
        ("kv_rank", C.c_uint32), ("rope_dim", C.c_uint32), ("quantized", C.c_uint32),
        ("nblk", C.c_uint32), ("device", C.c_int32), ("kv", C.c_void_p), ("pe", C.c_void_p),
        ("qs", C.c_void_p), ("sc", C.c_void_p), ("pool_bytes", C.c_uint64),
        ("checkpoint_bytes", C.c_uint64),
    ]


_lib = None

_u32, _u64, _i32, _i64, _f32, _vp = C.c_uint32, C.c_uint64, C.c_int, C.c_int64, C.c_float, C.c_void_p
_cp = C.c_char_p
_SIGS = {
    # device level
    "kvcu_get_last_error": (_cp, []),
    "kvcu_init": (_i32, [_i32]),
    "kvcu_device_count": (_i32, []),
    "kvcu_version": (_u32, []),
    "kvcu_pool_create": (_vp, [_i32, _u32, _u32, _u32, _u32, _u32, _i32]),
    "kvcu_pool_destroy": (_i32, [_vp]),
    "kvcu_pool_describe": (_i32, [_vp, C.POINTER(PoolDesc)]),
    "kvcu_pool_zero": (_i32, [_vp, _vp]),
    "kvcu_pool_status": (_i32, [_vp, C.POINTER(_u32), _vp]),
    "kvcu_pool_copy_block": (_i32, [_vp, _u32, _u32, _vp]),
    "kvcu_append": (_i32, [_vp, _u32, _u32, _vp, _u64, _vp, _u64, _vp, _vp, _u32, _vp, _vp, _vp, _vp]),
    "kvcu_append_layers": (_i32, [_vp, _u32, _u32, _u32, _vp, _u64, _u64, _vp, _u64, _u64, _vp, _vp, _u32, _vp, _vp,
                                  _vp, _vp]),
    "kvcu_gather": (_i32, [_vp, _u32, _vp, _u32, _u32, _vp, _vp]),
    "kvcu_gather_rows": (_i32, [_vp, _u32, _u32, _vp, _vp, _u32, _vp, _vp, _vp, _vp]),
    "kvcu_decode_ws_create": (_vp, [_i32, _u32, _u32]),
    "kvcu_decode_ws_create_layers": (_vp, [_i32, _u32, _u32, _u32]),
    "kvcu_mla_decode_layers": (_i32, [_vp, _vp, _u32, _u32, _u32, _vp, _u32, _vp, _vp, _vp, _vp, _u64, _u32, _f32,
                                      _vp, _u64, _vp]),
    "kvcu_decode_ws_destroy": (_i32, [_vp]),
    "kvcu_decode_plan": (_i32, [_vp, _vp, _u32, _vp, _u32, _vp, _vp]),
    "kvcu_decode_plan_causal": (_i32, [_vp, _vp, _u32, _vp, _u32, _vp, _vp, _vp]),
    "kvcu_decode_plan_layers": (_i32, [_vp, _vp, _u32, _vp, _u32, _vp, _u32, _vp]),
    "kvcu_mla_decode": (_i32, [_vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp, _vp, _u32, _f32, _vp, _vp]),
    "kvcu_mla_decode_lse": (_i32, [_vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp, _vp, _u32, _f32, _vp, _vp,
                                   _vp]),
    "kvcu_mla_prepare": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _f32, _f32, _vp, _vp, _vp, _vp]),
    "kvcu_mla_finish": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _f32, _vp, _vp, _vp]),
    "kvcu_decode_last_launches": (_u32, [_vp]),
    "kvcu_head_gemm": (_i32, [_i32, _u32, _u32, _u32, _u32, _vp, _u32, _u64, _vp, _u32, _u64, _vp, _u32, _u64, _i32,
                              _vp, _vp]),
    "kvcu_decode_ws_set_impl": (_i32, [_vp, _i32]),
    "kvcu_decode_ws_set_wait_limit": (_i32, [_vp, _u64]),
    "kvcu_decode_ws_test_withhold": (_i32, [_vp, _u32]),
    "kvcu_decode_last_impl": (_i32, [_vp]),
    "kvcu_mla_decode_noalloc": (_i32, [_vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp, _vp, _u32, _f32, _vp, _vp]),
    "kvcu_pool_read_checkpoint": (_i32, [_vp, _u64, _u64, _vp, _vp]),
    "kvcu_pool_write_checkpoint": (_i32, [_vp, _u64, _u64, _vp, _vp]),
    "kvcu_synth_rows": (_i32, [_u64, _u64, _u32, _vp, _vp, _u32, _f32, _vp, _vp]),
    # host mirror
    "kvcache_init": (_vp, [_i32, _u32, _u32, _u32, _u32, _u32]),
    "kvcache_init_blocks": (_vp, [_i32, _u32, _u32, _u32, _u32, _u32, _i32]),
    "kvcache_deinit": (None, [_vp]),
    "kvcache_enable_quantization": (_i32, [_vp]),
    "kvcache_ensure_capacity": (_i32, [_vp, _u32]),
    "kvcache_truncate": (None, [_vp, _u32]),
    "kvcache_reset": (None, [_vp]),
    "kvcache_put": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "kvcache_get_kv_compressed": (_i32, [_vp, _u32, _u32, _vp]),
    "kvcache_get_kpe": (_i32, [_vp, _u32, _u32, _vp]),
    "kvcache_len": (_u32, [_vp]),
    "kvcache_num_blocks": (_u32, [_vp]),
    "kvcache_block_size": (_u32, [_vp]),
    "kvcache_quantized": (_i32, [_vp]),
    "kvcache_num_free_blocks": (_u32, [_vp]),
    "kvcache_memory_usage": (_u64, [_vp]),
    "kvcache_block_table": (_u32, [_vp, _vp, _u32]),
    "kvcache_refcount": (_u32, [_vp, _u32]),
    "kvcache_set_free_list": (_i32, [_vp, _vp, _u32]),
    "kvcache_pool": (_vp, [_vp]),
    "kvcache_save_to_file": (_i32, [_vp, _cp]),
    "kvcache_load_from_file": (_i32, [_vp, _cp]),
    "kvcache_cache_block": (None, [_vp, _u32, _vp, _u32, _u64]),
    "kvcache_find_prefix_blocks": (_u32, [_vp, _vp, _u32]),
    "kvcache_reuse_prefix_blocks": (_i32, [_vp, _vp, _u32, _u32]),
    "kvcache_seq_cache_block": (_i32, [_vp, _u32, _u32, _vp, _u32, _u64]),
    "kvcache_seq_reuse_prefix_blocks": (_i32, [_vp, _u32, _vp, _u32, _u32]),
    "kvcache_compute_hash": (_u64, [_vp, _u32, _u64]),
    "kvcache_seq_create": (_i64, [_vp]),
    "kvcache_num_seqs": (_u32, [_vp]),
    "kvcache_seq_ensure_capacity": (_i32, [_vp, _u32, _u32]),
    "kvcache_seq_truncate": (_i32, [_vp, _u32, _u32]),
    "kvcache_seq_reset": (_i32, [_vp, _u32]),
    "kvcache_seq_len": (_u32, [_vp, _u32]),
    "kvcache_seq_block_table": (_u32, [_vp, _u32, _vp, _u32]),
    "kvcache_append_batch": (_i32, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "kvcache_append_batch_dev": (_i32, [_vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "kvcache_gather": (_i32, [_vp, _u32, _u32, _vp]),
    "kvcache_mla_decode": (_i32, [_vp, _u32, _u32, _vp, _vp, _u32, _f32, _vp]),
    "kvcache_mla_attention_batch": (_i32, [_vp, _u32, _u32, _u32, _u32, _vp, _u32, _f32, _vp]),
    "kvcache_mla_attention_batch_dev": (_i32, [_vp, _u32, _u32, _u32, _u32, _vp, _u32, _f32, _vp, _vp]),
    "kvcache_mla_decode_dev": (_i32, [_vp, _u32, _u32, _vp, _vp, _u32, _f32, _vp, _vp]),
    "kvcache_append_layers_dev": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _u64, _vp]),
    "kvcache_mla_decode_layers_dev": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp, _u64, _u32, _f32, _vp, _u64, _vp]),
    "kvcache_append_decode_layers": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _u32, _f32, _vp]),
    "kvcache_mla_step_dev": (_i32, [_vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _f32, _f32, _vp, _vp, _u32,
                                    _u32, _u32, _f32, _vp, _vp]),
    "kvcache_last_launches": (_u32, [_vp]),
    "kvcache_last_decode_mapped": (_i32, [_vp]),
    "kvcache_set_host_io": (_i32, [_vp, _i32]),
    "kvcache_set_decode_impl": (_i32, [_vp, _i32]),
    "kvcache_last_decode_impl": (_i32, [_vp]),
    "kvcache_save_to_file_v2": (_i32, [_vp, _cp]),
    "kvcache_load_from_file_v2": (_i32, [_vp, _cp]),
    "kvcache_save_to_file_v2_async": (_i32, [_vp, _cp, _vp, C.POINTER(_vp)]),
    "kvcache_save_done": (_i32, [_vp]),
    "kvcache_save_wait": (_i32, [_vp]),
    "kvcu_batch_create": (_vp, [_vp, _u32]),
    "kvcu_batch_destroy": (_i32, [_vp]),
    "kvcu_batch_add_request": (_i64, [_vp, _u32, _i32]),
    "kvcu_batch_collect": (_u32, [_vp, _u32, _vp, _vp, _u32]),
    "kvcu_batch_mark_running": (_i32, [_vp, _vp, _u32]),
    "kvcu_batch_mark_completed": (_i32, [_vp, _u64]),
    "kvcu_batch_set_status": (_i32, [_vp, _u64, _i32]),
    "kvcu_batch_status": (_i32, [_vp, _u64]),
    "kvcu_batch_push_token": (_i32, [_vp, _u64, _u32]),
    "kvcu_batch_is_finished": (_i32, [_vp, _u64, _u32]),
    "kvcu_batch_reap_completed": (_u32, [_vp]),
    "kvcu_batch_reclaim_blocks": (_u32, [_vp]),
    "kvcu_batch_running_count": (_u32, [_vp]),
    "kvcu_batch_size": (_u32, [_vp]),
    "kvcu_batch_seq": (_i64, [_vp, _u64]),
}


def lib():
    """Load libkvcuda.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python mobile-moe.zig_b200/build.py`"
                          " (the CUDA path has no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    return lib().kvcu_get_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise KVCudaError(rc, what, last_error())


def _np_ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _dptr(t) -> C.c_void_p:
    """Device pointer of a torch tensor (or an int address / None)."""
    if t is None:
        return C.c_void_p(0)
    if isinstance(t, int):
        return C.c_void_p(t)
    return C.c_void_p(t.data_ptr())


def _stream(s) -> C.c_void_p:
    if s is None:
        return C.c_void_p(0)
    if isinstance(s, int):
        return C.c_void_p(s)
    return C.c_void_p(s.cuda_stream)


def device_count() -> int:
    return lib().kvcu_device_count()


def init(device: int = 0) -> None:
    check(lib().kvcu_init(device), "kvcu_init")


# ------------------------------------------------------------------ device level
class DevicePool:
    """kvcu_pool: the physical block pool of one GPU (all layers)."""

    def __init__(self, device, n_layers, num_blocks, block_size, kv_rank, rope_dim, quantized):
        h = lib().kvcu_pool_create(device, n_layers, num_blocks, block_size, kv_rank, rope_dim,
                                   1 if quantized else 0)
        if not h:
            raise KVCudaError(-14, "kvcu_pool_create", last_error())
        self._h, self._own = h, True
        self.device = device

    @classmethod
    def borrow(cls, handle):
        self = cls.__new__(cls)
        self._h, self._own = handle, False
        self.device = self.describe().device
        return self

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None) and self._own:
            lib().kvcu_pool_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def describe(self) -> PoolDesc:
        d = PoolDesc()
        check(lib().kvcu_pool_describe(self._h, C.byref(d)), "kvcu_pool_describe")
        return d

    def status(self, stream=None) -> int:
        v = C.c_uint32(0)
        check(lib().kvcu_pool_status(self._h, C.byref(v), _stream(stream)), "kvcu_pool_status")
        return v.value

    def zero(self, stream=None):
        check(lib().kvcu_pool_zero(self._h, _stream(stream)), "kvcu_pool_zero")

    def append(self, layer, rows, row_seq, row_pos, table_offsets, tables, lens=None, stream=None,
               latent=None, latent_stride=None, rope=None, rope_stride=None):
        """rows: device f32 [n][kv_rank+rope_dim] (or explicit latent/rope pointers)."""
        d = self.describe()
        n = row_seq.numel()
        W = d.kv_rank + d.rope_dim
        if latent is None:
            latent = rows.data_ptr()
            rope = rows.data_ptr() + 4 * d.kv_rank
            latent_stride = rope_stride = W
        check(lib().kvcu_append(self._h, layer, n, C.c_void_p(latent), latent_stride, C.c_void_p(rope),
                                rope_stride, _dptr(row_seq), _dptr(row_pos), table_offsets.numel() - 1,
                                _dptr(table_offsets), _dptr(tables), _dptr(lens), _stream(stream)),
              "kvcu_append")

    def append_layers(self, layer, rows, row_seq, row_pos, table_offsets, tables, lens=None, stream=None):
        """rows: device f32 [n_layers][n][kv_rank+rope_dim]; one launch for layers [layer, layer+n_layers)."""
        d = self.describe()
        nl, n, W = rows.shape
        check(lib().kvcu_append_layers(self._h, layer, nl, n, C.c_void_p(rows.data_ptr()), W, n * W,
                                       C.c_void_p(rows.data_ptr() + 4 * d.kv_rank), W, n * W, _dptr(row_seq),
                                       _dptr(row_pos), table_offsets.numel() - 1, _dptr(table_offsets),
                                       _dptr(tables), _dptr(lens), _stream(stream)), "kvcu_append_layers")

    def gather(self, layer, table, length, out, stream=None):
        check(lib().kvcu_gather(self._h, layer, _dptr(table), table.numel(), length, _dptr(out),
                                _stream(stream)), "kvcu_gather")

    def gather_rows(self, layer, row_seq, row_pos, table_offsets, tables, out, stream=None):
        check(lib().kvcu_gather_rows(self._h, layer, row_seq.numel(), _dptr(row_seq), _dptr(row_pos),
                                     table_offsets.numel() - 1, _dptr(table_offsets), _dptr(tables),
                                     _dptr(out), _stream(stream)), "kvcu_gather_rows")

    def read_checkpoint(self, offset=0, nbytes=None, stream=None) -> bytes:
        d = self.describe()
        if nbytes is None:
            nbytes = d.checkpoint_bytes - offset
        buf = np.zeros(max(nbytes, 1), np.uint8)
        check(lib().kvcu_pool_read_checkpoint(self._h, offset, nbytes, _np_ptr(buf), _stream(stream)),
              "kvcu_pool_read_checkpoint")
        return buf[:nbytes].tobytes()

    def write_checkpoint(self, data: bytes, offset=0, stream=None):
        buf = np.frombuffer(data, np.uint8).copy() if data else np.zeros(1, np.uint8)
        check(lib().kvcu_pool_write_checkpoint(self._h, offset, len(data), _np_ptr(buf),
                                               _stream(stream)), "kvcu_pool_write_checkpoint")


class DecodeWorkspace:
    def __init__(self, device, max_batch, max_heads, max_layers=1):
        h = lib().kvcu_decode_ws_create_layers(device, max_batch, max_heads, max_layers)
        if not h:
            raise KVCudaError(-14, "kvcu_decode_ws_create", last_error())
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().kvcu_decode_ws_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def plan(self, pool: DevicePool, lens, seq_ids=None, n=None, stream=None):
        n = n if n is not None else (seq_ids.numel() if seq_ids is not None else lens.numel())
        check(lib().kvcu_decode_plan(self._h, pool.handle, n, _dptr(seq_ids), lens.numel(), _dptr(lens),
                                     _stream(stream)), "kvcu_decode_plan")

    def plan_layers(self, pool: DevicePool, lens, n_layers, seq_ids=None, n=None, stream=None):
        """One plan for a decode_layers call of n_layers layers (all (layer, entry) pairs balanced as one list)."""
        n = n if n is not None else (seq_ids.numel() if seq_ids is not None else lens.numel())
        check(lib().kvcu_decode_plan_layers(self._h, pool.handle, n, _dptr(seq_ids), lens.numel(), _dptr(lens),
                                            n_layers, _stream(stream)), "kvcu_decode_plan_layers")

    def decode(self, pool: DevicePool, layer, q, table_offsets, tables, lens, scale, out,
               seq_ids=None, stream=None):
        n, H = q.shape[0], q.shape[1]
        check(lib().kvcu_mla_decode(self._h, pool.handle, layer, n, _dptr(seq_ids), lens.numel(),
                                    _dptr(table_offsets), _dptr(tables), _dptr(lens), _dptr(q), H,
                                    scale, _dptr(out), _stream(stream)), "kvcu_mla_decode")

    def decode_layers(self, pool: DevicePool, layer, q, table_offsets, tables, lens, scale, out, seq_ids=None,
                      stream=None):
        """q [n_layers][n][H][576], out [n_layers][n][H][512]: layers [layer, layer+n_layers), one plan."""
        nl, n, H = q.shape[0], q.shape[1], q.shape[2]
        check(lib().kvcu_mla_decode_layers(self._h, pool.handle, layer, nl, n, _dptr(seq_ids), lens.numel(),
                                           _dptr(table_offsets), _dptr(tables), _dptr(lens), _dptr(q),
                                           q[0].numel(), H, scale, _dptr(out), out[0].numel(), _stream(stream)),
              "kvcu_mla_decode_layers")

    @property
    def last_launches(self):
        return lib().kvcu_decode_last_launches(self._h)

    def set_impl(self, impl):
        check(lib().kvcu_decode_ws_set_impl(self._h, impl), "kvcu_decode_ws_set_impl")

    def set_wait_limit(self, cycles):
        check(lib().kvcu_decode_ws_set_wait_limit(self._h, cycles), "kvcu_decode_ws_set_wait_limit")

    def test_withhold(self, tile):
        """Test hook: withhold the first slice of tile `tile` of every CTA (0xFFFFFFFF: off)."""
        check(lib().kvcu_decode_ws_test_withhold(self._h, tile), "kvcu_decode_ws_test_withhold")

    @property
    def last_impl(self):
        return lib().kvcu_decode_last_impl(self._h)


def synth_rows(seed, a, b, c, width, out, outlier_p=0.0, stream=None):
    """out[r][i] = N(0,1)(seed, a, b[r], c[r]*1024+i) on the device (b, c, out: CUDA tensors)."""
    check(lib().kvcu_synth_rows(seed, a, b.numel(), _dptr(b), _dptr(c), width, outlier_p, _dptr(out),
                                _stream(stream)), "kvcu_synth_rows")


def prefill_synthetic(pool: DevicePool, layer, lens, table_offsets, tables, seed, outlier_p=0.0,
                      gen_layer=None, seq_tags=None, lens_dev=None, chunk_rows=1 << 16,
                      stream=None, start=None):
    """Append positions [start[s], lens[s]) of every sequence s with the seeded
    generator's rows (gen tag `gen_layer`, default `layer`; row of sequence s at
    position t = normal(seed, tag, seq_tags[s], t*1024 + i)).  Everything runs on
    the device; returns the number of rows appended."""
    import torch

    d = pool.describe()
    W = d.kv_rank + d.rope_dim
    dev = torch.device("cuda", pool.device)
    lens = np.asarray(lens, np.int64)
    start = np.zeros_like(lens) if start is None else np.asarray(start, np.int64)
    tags = np.arange(lens.size, dtype=np.int64) if seq_tags is None else np.asarray(seq_tags, np.int64)
    counts = np.maximum(lens - start, 0)
    total = int(counts.sum())
    if total == 0:
        return 0
    seq_of = np.repeat(np.arange(lens.size, dtype=np.uint32), counts)
    pos_of = (np.arange(total, dtype=np.int64) - np.repeat(np.cumsum(counts) - counts, counts)
              + np.repeat(start, counts)).astype(np.uint32)
    tag_of = tags.astype(np.uint32)[seq_of]
    rows = torch.empty((min(chunk_rows, total), W), dtype=torch.float32, device=dev)
    g = layer if gen_layer is None else gen_layer
    for k in range(0, total, chunk_rows):
        n = min(chunk_rows, total - k)
        s_d = torch.from_numpy(seq_of[k:k + n].copy()).to(dev)
        p_d = torch.from_numpy(pos_of[k:k + n].copy()).to(dev)
        t_d = torch.from_numpy(tag_of[k:k + n].copy()).to(dev)
        synth_rows(seed, g, t_d, p_d, W, rows[:n], outlier_p, stream)
        pool.append(layer, rows[:n], s_d, p_d, table_offsets, tables, lens=lens_dev, stream=stream)
    return total


# ------------------------------------------------------------------ host mirror
class KVCache:
    """mobile-moe.zig's KVCache (src/kv_cache.zig) on a B200, plus many sequences.

    KVCache(n_layers, kv_rank, rope_dim, max_seq_len, block_size=16, device=0) is
    KVCache.init(allocator, hp, max_seq_len).  Use KVCache.with_blocks(...) for a
    pool shared by many sequences.
    """

    def __init__(self, n_layers, kv_rank, rope_dim, max_seq_len, block_size=16, device=0,
                 _handle=None):
        h = _handle or lib().kvcache_init(device, n_layers, kv_rank, rope_dim, max_seq_len, block_size)
        if not h:
            raise KVCudaError(-14, "kvcache_init", last_error())
        self._h = h
        self.kv_rank, self.rope_dim, self.n_layers, self.device = kv_rank, rope_dim, n_layers, device

    @classmethod
    def with_blocks(cls, n_layers, kv_rank, rope_dim, num_blocks, block_size=16, quantized=False,
                    device=0):
        h = lib().kvcache_init_blocks(device, n_layers, kv_rank, rope_dim, num_blocks, block_size,
                                      1 if quantized else 0)
        if not h:
            raise KVCudaError(-14, "kvcache_init_blocks", last_error())
        return cls(n_layers, kv_rank, rope_dim, 0, block_size, device, _handle=h)

    def deinit(self):
        if getattr(self, "_h", None):
            lib().kvcache_deinit(self._h)
        self._h = None

    close = deinit

    def __del__(self):
        try:
            self.deinit()
        except Exception:
            pass

    # ---- reference API (src/kv_cache.zig) ----
    def enableQuantization(self):
        check(lib().kvcache_enable_quantization(self._h), "enableQuantization")

    def ensureCapacity(self, n_tokens):
        check(lib().kvcache_ensure_capacity(self._h, n_tokens), "ensureCapacity")

    def truncate(self, n_tokens):
        lib().kvcache_truncate(self._h, n_tokens)

    def reset(self):
        lib().kvcache_reset(self._h)

    def put(self, layer, pos, kv_comp, k_pe):
        a = np.ascontiguousarray(kv_comp, np.float32)
        b = np.ascontiguousarray(k_pe, np.float32)
        assert a.size == self.kv_rank and b.size == self.rope_dim
        check(lib().kvcache_put(self._h, layer, pos, _np_ptr(a), _np_ptr(b)), "put")

    def getKVCompressed(self, layer, pos):
        out = np.zeros(self.kv_rank, np.float32)
        check(lib().kvcache_get_kv_compressed(self._h, layer, pos, _np_ptr(out)), "getKVCompressed")
        return out

    def getKPe(self, layer, pos):
        out = np.zeros(self.rope_dim, np.float32)
        check(lib().kvcache_get_kpe(self._h, layer, pos, _np_ptr(out)), "getKPe")
        return out

    @property
    def len(self):
        return lib().kvcache_len(self._h)

    @property
    def num_blocks(self):
        return lib().kvcache_num_blocks(self._h)

    @property
    def block_size(self):
        return lib().kvcache_block_size(self._h)

    @property
    def quantized(self):
        return bool(lib().kvcache_quantized(self._h))

    @property
    def block_table(self):
        return self.seq_block_table(0)

    def numFreeBlocks(self):
        return lib().kvcache_num_free_blocks(self._h)

    def memoryUsage(self):
        return lib().kvcache_memory_usage(self._h)

    def refcount(self, block_id):
        return lib().kvcache_refcount(self._h, block_id)

    def set_free_list(self, ids):
        ids = np.ascontiguousarray(ids, np.uint32)
        check(lib().kvcache_set_free_list(self._h, _np_ptr(ids), ids.size), "set_free_list")

    def pool(self) -> DevicePool:
        return DevicePool.borrow(lib().kvcache_pool(self._h))

    def saveToFile(self, path):
        check(lib().kvcache_save_to_file(self._h, os.fsencode(str(path))), "saveToFile")

    def loadFromFile(self, path):
        check(lib().kvcache_load_from_file(self._h, os.fsencode(str(path))), "loadFromFile")

    def saveToFileV2(self, path):
        check(lib().kvcache_save_to_file_v2(self._h, os.fsencode(str(path))), "saveToFileV2")

    def loadFromFileV2(self, path):
        check(lib().kvcache_load_from_file_v2(self._h, os.fsencode(str(path))), "loadFromFileV2")

    def saveToFileV2Async(self, path, stream=None) -> "SaveJob":
        """Background v2 save of the cache as it is now (kvcache_save_to_file_v2_async);
        serving may go on; .wait() returns when the file is complete."""
        h = C.c_void_p()
        check(lib().kvcache_save_to_file_v2_async(self._h, os.fsencode(str(path)), _stream(stream), C.byref(h)),
              "saveToFileV2Async")
        return SaveJob(h.value)

    def cacheBlock(self, block_idx, token_ids, prefix_hash):
        t = np.ascontiguousarray(token_ids, np.uint32)
        lib().kvcache_cache_block(self._h, block_idx, _np_ptr(t), t.size, prefix_hash)

    def findPrefixBlocks(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        return lib().kvcache_find_prefix_blocks(self._h, _np_ptr(t), t.size)

    def reusePrefixBlocks(self, tokens, n_blocks):
        t = np.ascontiguousarray(tokens, np.uint32)
        check(lib().kvcache_reuse_prefix_blocks(self._h, _np_ptr(t), t.size, n_blocks),
              "reusePrefixBlocks")

    def seq_cache_block(self, seq, block_idx, token_ids, prefix_hash):
        t = np.ascontiguousarray(token_ids, np.uint32)
        check(lib().kvcache_seq_cache_block(self._h, seq, block_idx, _np_ptr(t), t.size, prefix_hash),
              "seq_cache_block")

    def seq_reuse_prefix_blocks(self, seq, tokens, n_blocks):
        t = np.ascontiguousarray(tokens, np.uint32)
        check(lib().kvcache_seq_reuse_prefix_blocks(self._h, seq, _np_ptr(t), t.size, n_blocks),
              "seq_reuse_prefix_blocks")

    @staticmethod
    def computeHash(token_ids, prefix_hash=NO_HASH):
        t = np.ascontiguousarray(token_ids, np.uint32)
        if t.size == 0:
            t = np.zeros(1, np.uint32)
            return lib().kvcache_compute_hash(_np_ptr(t), 0, prefix_hash)
        return lib().kvcache_compute_hash(_np_ptr(t), t.size, prefix_hash)

    # ---- many sequences ----
    def seq_create(self) -> int:
        r = lib().kvcache_seq_create(self._h)
        if r < 0:
            check(int(r), "seq_create")
        return int(r)

    @property
    def num_seqs(self):
        return lib().kvcache_num_seqs(self._h)

    def seq_ensure_capacity(self, seq, n_tokens):
        check(lib().kvcache_seq_ensure_capacity(self._h, seq, n_tokens), "seq_ensure_capacity")

    def seq_truncate(self, seq, n_tokens):
        check(lib().kvcache_seq_truncate(self._h, seq, n_tokens), "seq_truncate")

    def seq_reset(self, seq):
        check(lib().kvcache_seq_reset(self._h, seq), "seq_reset")

    def seq_len(self, seq):
        return lib().kvcache_seq_len(self._h, seq)

    def seq_block_table(self, seq):
        n = lib().kvcache_seq_block_table(self._h, seq, None, 0)
        out = np.zeros(max(n, 1), np.uint32)
        lib().kvcache_seq_block_table(self._h, seq, _np_ptr(out), n)
        return [int(x) for x in out[:n]]

    def appendBatch(self, layer, seq_ids, positions, rows):
        s = np.ascontiguousarray(seq_ids, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        r = np.ascontiguousarray(rows, np.float32)
        assert r.shape == (s.size, self.kv_rank + self.rope_dim)
        check(lib().kvcache_append_batch(self._h, layer, s.size, _np_ptr(s), _np_ptr(p), _np_ptr(r)),
              "appendBatch")

    def appendBatch_dev(self, layer, seq_ids, positions, seq_ids_dev, positions_dev, rows_dev,
                        stream=None):
        s = np.ascontiguousarray(seq_ids, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        check(lib().kvcache_append_batch_dev(self._h, layer, s.size, _np_ptr(s), _np_ptr(p),
                                             _dptr(seq_ids_dev), _dptr(positions_dev), _dptr(rows_dev),
                                             _stream(stream)), "appendBatch_dev")

    def appendLayers_dev(self, layer, seq_ids, positions, seq_ids_dev, positions_dev, rows_dev, stream=None):
        """rows_dev [n_layers][n][W]: appendBatch of layers [layer, layer+n_layers) in one launch."""
        s = np.ascontiguousarray(seq_ids, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        nl = rows_dev.shape[0]
        check(lib().kvcache_append_layers_dev(self._h, layer, nl, s.size, _np_ptr(s), _np_ptr(p), _dptr(seq_ids_dev),
                                              _dptr(positions_dev), _dptr(rows_dev), rows_dev[0].numel(),
                                              _stream(stream)), "appendLayers_dev")

    def mlaDecodeLayers_dev(self, layer, seq_ids, q_dev, scale, out_dev, stream=None):
        """q_dev [n_layers][n][H][W] -> out_dev [n_layers][n][H][R], one multi-layer launch."""
        s = np.ascontiguousarray(seq_ids, np.uint32)
        nl, n, H = q_dev.shape[0], q_dev.shape[1], q_dev.shape[2]
        check(lib().kvcache_mla_decode_layers_dev(self._h, layer, nl, n, _np_ptr(s), _dptr(q_dev), q_dev[0].numel(),
                                                  H, scale, _dptr(out_dev), out_dev[0].numel(), _stream(stream)),
              "mlaDecodeLayers_dev")

    def appendDecodeLayers_ptr(self, layer, n_layers, n, seq_ids, positions, rows_ptr, q_ptr, n_heads, scale,
                               out_ptr):
        """Host buffers (raw addresses): rows [nl][n][W], q [nl][n][H][W] -> out [nl][n][H][R]; one sync."""
        s = np.ascontiguousarray(seq_ids, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        check(lib().kvcache_append_decode_layers(self._h, layer, n_layers, n, _np_ptr(s), _np_ptr(p),
                                                 C.c_void_p(rows_ptr), C.c_void_p(q_ptr), n_heads, scale,
                                                 C.c_void_p(out_ptr)), "appendDecodeLayers")

    def gather(self, layer, seq):
        n = self.seq_len(seq)
        out = np.zeros((max(n, 1), self.kv_rank + self.rope_dim), np.float32)
        check(lib().kvcache_gather(self._h, layer, seq, _np_ptr(out)), "gather")
        return out[:n]

    def mlaDecode(self, layer, q, seq_ids, scale, out=None):
        """q: host f32 [n][H][kv_rank+rope_dim] -> out host f32 [n][H][kv_rank]."""
        q = np.ascontiguousarray(q, np.float32)
        s = np.ascontiguousarray(seq_ids, np.uint32)
        n, H = q.shape[0], q.shape[1]
        if out is None:
            out = np.zeros((n, H, self.kv_rank), np.float32)
        check(lib().kvcache_mla_decode(self._h, layer, n, _np_ptr(s), _np_ptr(q), H, scale,
                                       _np_ptr(out)), "mlaDecode")
        return out

    def mlaAttentionBatch(self, layer, seq, start_pos, q, scale, out=None):
        """mlaAttentionBatch (src/inference.zig:670-883): host q [n_pos][H][W] for positions
        start_pos.. of `seq`, each attending causally -> out host [n_pos][H][kv_rank]."""
        q = np.ascontiguousarray(q, np.float32)
        n, H = q.shape[0], q.shape[1]
        if out is None:
            out = np.zeros((n, H, self.kv_rank), np.float32)
        check(lib().kvcache_mla_attention_batch(self._h, layer, seq, start_pos, n, _np_ptr(q), H, scale,
                                                _np_ptr(out)), "mlaAttentionBatch")
        return out

    def mlaAttentionBatch_dev(self, layer, seq, start_pos, q_dev, scale, out_dev, stream=None):
        n, H = q_dev.shape[0], q_dev.shape[1]
        check(lib().kvcache_mla_attention_batch_dev(self._h, layer, seq, start_pos, n, _dptr(q_dev), H, scale,
                                                    _dptr(out_dev), _stream(stream)), "mlaAttentionBatch_dev")

    def mlaDecode_ptr(self, layer, n, seq_ids, q_ptr, n_heads, scale, out_ptr):
        """Host-buffer decode on raw host addresses (pinned buffers for the e2e path)."""
        check(lib().kvcache_mla_decode(self._h, layer, n, _np_ptr(seq_ids), C.c_void_p(q_ptr), n_heads,
                                       scale, C.c_void_p(out_ptr)), "mlaDecode")

    def mlaDecode_dev(self, layer, seq_ids, q_dev, scale, out_dev, stream=None):
        s = np.ascontiguousarray(seq_ids, np.uint32)
        n, H = q_dev.shape[0], q_dev.shape[1]
        check(lib().kvcache_mla_decode_dev(self._h, layer, n, _np_ptr(s), _dptr(q_dev), H, scale,
                                           _dptr(out_dev), _stream(stream)), "mlaDecode_dev")

    def mla_step_dev(self, layer, seq_ids, positions, q, kv_a, norm_w, eps, rope_base, k_b, v_b, qk_nope, v_dim,
                     scale, attn, stream=None):
        """One MLA decode step (kvcache_mla_step_dev): device tensors q [n][H][qk_nope+P],
        kv_a [n][R+P], norm_w [R], k_b [H*qk_nope][R], v_b [H*v_dim][R] -> attn [n][H][v_dim]."""
        s = np.ascontiguousarray(seq_ids, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        n, H = q.shape[0], q.shape[1]
        check(lib().kvcache_mla_step_dev(self._h, layer, n, _np_ptr(s), _np_ptr(p), _dptr(q), _dptr(kv_a),
                                         _dptr(norm_w), eps, rope_base, _dptr(k_b), _dptr(v_b), H, qk_nope,
                                         v_dim, scale, _dptr(attn), _stream(stream)), "mla_step_dev")

    @property
    def last_launches(self):
        return lib().kvcache_last_launches(self._h)

    @property
    def last_decode_mapped(self):
        """True when the last host-buffer decode used pinned, mapped q / out in place."""
        return bool(lib().kvcache_last_decode_mapped(self._h))

    def set_decode_impl(self, impl):
        check(lib().kvcache_set_decode_impl(self._h, impl), "set_decode_impl")

    HOST_IO_AUTO, HOST_IO_COPY, HOST_IO_COPY_IN = 0, 1, 2

    def set_host_io(self, mode):
        """kvcache_set_host_io: HOST_IO_AUTO (q / out in place over PCIe when pinned
        and mapped), HOST_IO_COPY (DMA copies around the kernels) or HOST_IO_COPY_IN
        (q by DMA, out in place; the multi-layer call)."""
        check(lib().kvcache_set_host_io(self._h, mode), "set_host_io")

    @property
    def last_decode_impl(self):
        return lib().kvcache_last_decode_impl(self._h)

    def prefill_synthetic(self, layer, seqs, lens, seed, outlier_p=0.0, seq_tags=None,
                          chunk_rows=1 << 16, stream=None, start=None):
        """Append positions [start[i], lens[i]) of sequences `seqs` on layer `layer`
        with the seeded generator (row of sequence i at position t =
        normal(seed, layer, seq_tags[i], t*1024 + j)); all on the device.  Returns
        the rows appended."""
        import torch

        W = self.kv_rank + self.rope_dim
        dev = torch.device("cuda", self.device)
        # run on torch's current stream, so the caching allocator's reuse of the
        # per-chunk index tensors stays ordered after the kernels that read them
        assert stream is None or stream == torch.cuda.current_stream(dev)
        stream = torch.cuda.current_stream(dev)
        seqs = np.asarray(seqs, np.int64)
        lens = np.asarray(lens, np.int64)
        start = np.zeros_like(lens) if start is None else np.asarray(start, np.int64)
        tags = seqs if seq_tags is None else np.asarray(seq_tags, np.int64)
        counts = np.maximum(lens - start, 0)
        total = int(counts.sum())
        if total == 0:
            return 0
        idx = np.repeat(np.arange(seqs.size), counts)
        pos_of = (np.arange(total, dtype=np.int64) - np.repeat(np.cumsum(counts) - counts, counts)
                  + np.repeat(start, counts)).astype(np.uint32)
        seq_of = seqs.astype(np.uint32)[idx]
        tag_of = tags.astype(np.uint32)[idx]
        rows = torch.empty((min(chunk_rows, total), W), dtype=torch.float32, device=dev)
        for k in range(0, total, chunk_rows):
            n = min(chunk_rows, total - k)
            s_h, p_h = seq_of[k:k + n].copy(), pos_of[k:k + n].copy()
            s_d = torch.from_numpy(s_h).to(dev)
            p_d = torch.from_numpy(p_h).to(dev)
            t_d = torch.from_numpy(tag_of[k:k + n].copy()).to(dev)
            synth_rows(seed, layer, t_d, p_d, W, rows[:n], outlier_p, stream)
            self.appendBatch_dev(layer, s_h, p_h, s_d, p_d, rows[:n], stream)
        return total


class SaveJob:
    """A background checkpoint save (kvcache_save_to_file_v2_async)."""

    def __init__(self, handle):
        self._h = handle

    def done(self) -> bool:
        return bool(lib().kvcache_save_done(self._h))

    def wait(self):
        if self._h:
            h, self._h = self._h, None
            check(lib().kvcache_save_wait(h), "kvcache_save_wait")


SEQ_WAITING, SEQ_RUNNING, SEQ_PAUSED, SEQ_COMPLETED = 0, 1, 2, 3
PRIORITY_LOW, PRIORITY_NORMAL, PRIORITY_HIGH, PRIORITY_CRITICAL = 0, 1, 2, 3


class BatchScheduler:
    """BatchScheduler (src/batch_queue.zig:75-232) over one KVCache's shared pool
    (kvcu_batch_*): each request is a sequence of `cache`."""

    def __init__(self, cache: "KVCache", max_batch_size: int):
        self._cache = cache  # keeps the cache alive while the scheduler uses it
        self._h = lib().kvcu_batch_create(cache._h, max_batch_size)
        if not self._h:
            raise KVCudaError(-11, "kvcu_batch_create", last_error())
        self.max_batch_size = max_batch_size

    def close(self):
        if getattr(self, "_h", None):
            lib().kvcu_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def addRequest(self, max_tokens, priority=PRIORITY_NORMAL) -> int:
        rc = lib().kvcu_batch_add_request(self._h, max_tokens, priority)
        if rc < 0:
            check(int(rc), "addRequest")
        return int(rc)

    def collectBatch(self, eos_token=0):
        """(ids, pool sequences) of the next batch, in priority then arrival order."""
        ids = np.zeros(self.max_batch_size, np.uint64)
        seqs = np.zeros(self.max_batch_size, np.uint32)
        n = lib().kvcu_batch_collect(self._h, eos_token, _np_ptr(ids), _np_ptr(seqs), self.max_batch_size)
        return ids[:n].copy(), seqs[:n].copy()

    def markRunning(self, ids):
        a = np.ascontiguousarray(ids, np.uint64)
        check(lib().kvcu_batch_mark_running(self._h, _np_ptr(a), a.size), "markRunning")

    def markCompleted(self, rid):
        check(lib().kvcu_batch_mark_completed(self._h, rid), "markCompleted")

    def setStatus(self, rid, status):
        check(lib().kvcu_batch_set_status(self._h, rid, status), "setStatus")

    def status(self, rid) -> int:
        return lib().kvcu_batch_status(self._h, rid)

    def pushToken(self, rid, token):
        check(lib().kvcu_batch_push_token(self._h, rid, token), "pushToken")

    def isFinished(self, rid, eos_token=0) -> bool:
        rc = lib().kvcu_batch_is_finished(self._h, rid, eos_token)
        if rc < 0:
            check(rc, "isFinished")
        return bool(rc)

    def reapCompleted(self) -> int:
        return lib().kvcu_batch_reap_completed(self._h)

    def reclaimBlocks(self) -> int:
        return lib().kvcu_batch_reclaim_blocks(self._h)

    def runningCount(self) -> int:
        return lib().kvcu_batch_running_count(self._h)

    def __len__(self):
        return lib().kvcu_batch_size(self._h)

    def seq(self, rid) -> int:
        rc = lib().kvcu_batch_seq(self._h, rid)
        if rc < 0:
            check(int(rc), "seq")
        return int(rc)
