"""ctypes binding of the CPU oracle (oracle/libkvoracle.so).

TEST INFRASTRUCTURE ONLY.  The oracle is the parity checker for the CUDA
product; only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline
leg may import this module.  The product package never imports it.

The C library restates the reference's KV-cache hot path (see kvoracle.h for
the file:line list and the documented deviations).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkvoracle.so")

OK = 0
ERR_OUT_OF_BLOCKS = -1
ERR_POSITION_OOB = -2
ERR_LAYER_OOB = -3
ERR_POSITION_NOT_WRITTEN = -4
ERR_PREFIX_MISS = -5
ERR_BAD_MAGIC = -6
ERR_BAD_VERSION = -7
ERR_SHAPE_MISMATCH = -8
ERR_EOF = -9
ERR_IO = -10
ERR_INVALID_ARG = -11
ERR_NO_MEMORY = -14
ERR_BAD_BLOCK_ID = -15

NO_HASH = (1 << 64) - 1


def build() -> str:
    """Compile the oracle library (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _Pool(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("num_blocks", C.c_uint32), ("block_size", C.c_uint32),
        ("kv_rank", C.c_uint32), ("rope_dim", C.c_uint32), ("quantized", C.c_int),
        ("kv", C.c_void_p), ("pe", C.c_void_p), ("kv_q8", C.c_void_p), ("pe_q8", C.c_void_p),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        u32, u64, f32, i32, vp = C.c_uint32, C.c_uint64, C.c_float, C.c_int, C.c_void_p
        P = C.POINTER(_Pool)
        sig = {
            "kvo_f16_to_f32": (f32, [C.c_uint16]),
            "kvo_f32_to_f16": (C.c_uint16, [f32]),
            "kvo_quantize_q8_0": (None, [vp, u32, vp]),
            "kvo_dequantize_q8_0": (None, [vp, u32, vp]),
            "kvo_pool_init": (i32, [P, u32, u32, u32, u32, u32, i32]),
            "kvo_pool_free": (None, [P]),
            "kvo_pool_put": (None, [P, u32, u32, u32, vp, vp]),
            "kvo_pool_get": (None, [P, u32, u32, u32, vp, vp]),
            "kvo_pool_put_rows": (None, [P, u32, u32, vp, vp, vp]),
            "kvo_pool_gather": (None, [P, u32, vp, u32, vp]),
            "kvo_pool_bytes": (u64, [P]),
            "kvo_pool_serialize": (None, [P, vp]),
            "kvo_pool_deserialize": (None, [P, vp]),
            "kvo_attention": (None, [P, u32, vp, u32, vp, u32, f32, vp]),
            "kvo_attention_batch": (None, [P, u32, u32, vp, vp, vp, vp, u32, f32, vp, i32]),
            "kvo_cache_init": (vp, [u32, u32, u32, u32, u32]),
            "kvo_cache_deinit": (None, [vp]),
            "kvo_cache_enable_quantization": (i32, [vp]),
            "kvo_cache_ensure_capacity": (i32, [vp, u32]),
            "kvo_cache_truncate": (None, [vp, u32]),
            "kvo_cache_reset": (None, [vp]),
            "kvo_cache_put": (i32, [vp, u32, u32, vp, vp]),
            "kvo_cache_get_kv_compressed": (i32, [vp, u32, u32, vp]),
            "kvo_cache_get_kpe": (i32, [vp, u32, u32, vp]),
            "kvo_cache_len": (u32, [vp]),
            "kvo_cache_num_blocks": (u32, [vp]),
            "kvo_cache_num_free_blocks": (u32, [vp]),
            "kvo_cache_quantized": (i32, [vp]),
            "kvo_cache_block_table_len": (u32, [vp]),
            "kvo_cache_block_table": (C.POINTER(u32), [vp]),
            "kvo_cache_refcount": (u32, [vp, u32]),
            "kvo_cache_memory_usage": (u64, [vp]),
            "kvo_cache_pool": (P, [vp]),
            "kvo_cache_set_free_list": (i32, [vp, vp, u32]),
            "kvo_cache_save": (i32, [vp, C.c_char_p]),
            "kvo_cache_load": (i32, [vp, C.c_char_p]),
            "kvo_cache_cache_block": (None, [vp, u32, vp, u32, u64]),
            "kvo_cache_find_prefix_blocks": (u32, [vp, vp, u32]),
            "kvo_cache_reuse_prefix_blocks": (i32, [vp, vp, u32, u32]),
            "kvo_xxh64": (u64, [vp, C.c_size_t, u64]),
            "kvo_compute_hash": (u64, [vp, u32, u64]),
            "kvo_splitmix64": (u64, [u64]),
            "kvo_log_det": (f32, [f32]),
            "kvo_gen_normal": (f32, [u64, u64, u64, u64, f32]),
            "kvo_gen_rows": (None, [u64, u64, u32, vp, vp, u32, f32, vp, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- numerics
def f16_to_f32(h: int) -> float:
    return lib().kvo_f16_to_f32(h)


def f32_to_f16(v: float) -> int:
    return lib().kvo_f32_to_f16(v)


BLOCK_Q8_DTYPE = np.dtype([("d", "<u2"), ("qs", "i1", (32,))])
assert BLOCK_Q8_DTYPE.itemsize == 34


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros((x.size + 31) // 32, dtype=BLOCK_Q8_DTYPE)
    lib().kvo_quantize_q8_0(_ptr(x), x.size, _ptr(out))
    return out


def dequantize_q8_0(blocks: np.ndarray, n: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks)
    out = np.zeros(n, dtype=np.float32)
    lib().kvo_dequantize_q8_0(_ptr(blocks), n, _ptr(out))
    return out


# ---------------------------------------------------------------- pool
class Pool:
    """Reference-layout block pool ([L][NB][BS][...], separate kv / pe arrays)."""

    def __init__(self, n_layers, num_blocks, block_size, kv_rank, rope_dim, quantized):
        self._p = _Pool()
        rc = lib().kvo_pool_init(C.byref(self._p), n_layers, num_blocks, block_size, kv_rank,
                                 rope_dim, 1 if quantized else 0)
        if rc != OK:
            raise MemoryError(f"kvo_pool_init failed: {rc}")
        self.n_layers, self.num_blocks, self.block_size = n_layers, num_blocks, block_size
        self.kv_rank, self.rope_dim, self.quantized = kv_rank, rope_dim, bool(quantized)

    def __del__(self):
        if getattr(self, "_p", None) is not None and lib is not None:
            lib().kvo_pool_free(C.byref(self._p))
            self._p = None

    @property
    def ref(self):
        return C.byref(self._p)

    def put(self, layer, block, offset, kv_comp, k_pe):
        kv_comp = np.ascontiguousarray(kv_comp, np.float32)
        k_pe = np.ascontiguousarray(k_pe, np.float32)
        lib().kvo_pool_put(self.ref, layer, block, offset, _ptr(kv_comp), _ptr(k_pe))

    def put_rows(self, layer, blocks, offsets, rows):
        """rows: [n][kv_rank+rope_dim] written to (blocks[r], offsets[r])."""
        rows = np.ascontiguousarray(rows, np.float32)
        blocks = np.ascontiguousarray(blocks, np.uint32)
        offsets = np.ascontiguousarray(offsets, np.uint32)
        assert rows.shape == (blocks.size, self.kv_rank + self.rope_dim)
        lib().kvo_pool_put_rows(self.ref, layer, blocks.size, _ptr(blocks), _ptr(offsets), _ptr(rows))

    def get(self, layer, block, offset):
        kv = np.zeros(self.kv_rank, np.float32)
        pe = np.zeros(self.rope_dim, np.float32)
        lib().kvo_pool_get(self.ref, layer, block, offset, _ptr(kv), _ptr(pe))
        return kv, pe

    def gather(self, layer, table, length):
        table = np.ascontiguousarray(table, np.uint32)
        out = np.zeros((length, self.kv_rank + self.rope_dim), np.float32)
        lib().kvo_pool_gather(self.ref, layer, _ptr(table), length, _ptr(out))
        return out

    def serialize(self) -> bytes:
        n = lib().kvo_pool_bytes(self.ref)
        buf = np.zeros(n, np.uint8)
        lib().kvo_pool_serialize(self.ref, _ptr(buf))
        return buf.tobytes()

    def deserialize(self, data: bytes):
        buf = np.frombuffer(data, np.uint8).copy()
        assert buf.size == lib().kvo_pool_bytes(self.ref)
        lib().kvo_pool_deserialize(self.ref, _ptr(buf))

    def kv_q8_blocks(self) -> np.ndarray:
        """The Q8_0 latent pool as a [rows][ceil(kv_rank/32)] BlockQ8_0 array (copy)."""
        data = self.serialize()
        rows = self.n_layers * self.num_blocks * self.block_size
        nkv, npe = (self.kv_rank + 31) // 32, (self.rope_dim + 31) // 32
        a = np.frombuffer(data, BLOCK_Q8_DTYPE, count=rows * nkv).reshape(rows, nkv)
        b = np.frombuffer(data, BLOCK_Q8_DTYPE, offset=rows * nkv * 34, count=rows * npe)
        return a.copy(), b.reshape(rows, npe).copy()

    def attention(self, layer, table, length, q, scale):
        table = np.ascontiguousarray(table, np.uint32)
        q = np.ascontiguousarray(q, np.float32)
        H = q.shape[0]
        out = np.zeros((H, self.kv_rank), np.float32)
        lib().kvo_attention(self.ref, layer, _ptr(table), length, _ptr(q), H, scale, _ptr(out))
        return out

    def attention_batch(self, layer, table_offsets, tables, lens, q, scale, n_threads=1):
        table_offsets = np.ascontiguousarray(table_offsets, np.uint32)
        tables = np.ascontiguousarray(tables, np.uint32)
        lens = np.ascontiguousarray(lens, np.uint32)
        q = np.ascontiguousarray(q, np.float32)
        B, H = q.shape[0], q.shape[1]
        out = np.zeros((B, H, self.kv_rank), np.float32)
        lib().kvo_attention_batch(self.ref, layer, B, _ptr(table_offsets), _ptr(tables),
                                  _ptr(lens), _ptr(q), H, scale, _ptr(out), n_threads)
        return out


# ---------------------------------------------------------------- KVCache
class KVCache:
    """Single-sequence KVCache with the reference's method names (src/kv_cache.zig)."""

    def __init__(self, n_layers, kv_rank, rope_dim, max_seq_len, block_size=16):
        self._h = lib().kvo_cache_init(n_layers, kv_rank, rope_dim, max_seq_len, block_size)
        if not self._h:
            raise ValueError("kvo_cache_init failed")
        self.kv_rank, self.rope_dim = kv_rank, rope_dim

    def __del__(self):
        if getattr(self, "_h", None):
            lib().kvo_cache_deinit(self._h)
            self._h = None

    def enableQuantization(self):
        return lib().kvo_cache_enable_quantization(self._h)

    def ensureCapacity(self, n):
        return lib().kvo_cache_ensure_capacity(self._h, n)

    def truncate(self, n):
        lib().kvo_cache_truncate(self._h, n)

    def reset(self):
        lib().kvo_cache_reset(self._h)

    def put(self, layer, pos, kv_comp, k_pe):
        kv_comp = np.ascontiguousarray(kv_comp, np.float32)
        k_pe = np.ascontiguousarray(k_pe, np.float32)
        return lib().kvo_cache_put(self._h, layer, pos, _ptr(kv_comp), _ptr(k_pe))

    def getKVCompressed(self, layer, pos):
        out = np.zeros(self.kv_rank, np.float32)
        rc = lib().kvo_cache_get_kv_compressed(self._h, layer, pos, _ptr(out))
        return rc, out

    def getKPe(self, layer, pos):
        out = np.zeros(self.rope_dim, np.float32)
        rc = lib().kvo_cache_get_kpe(self._h, layer, pos, _ptr(out))
        return rc, out

    @property
    def len(self):
        return lib().kvo_cache_len(self._h)

    @property
    def num_blocks(self):
        return lib().kvo_cache_num_blocks(self._h)

    @property
    def quantized(self):
        return bool(lib().kvo_cache_quantized(self._h))

    @property
    def block_table(self):
        n = lib().kvo_cache_block_table_len(self._h)
        p = lib().kvo_cache_block_table(self._h)
        return [p[i] for i in range(n)]

    def numFreeBlocks(self):
        return lib().kvo_cache_num_free_blocks(self._h)

    def refcount(self, block_id):
        return lib().kvo_cache_refcount(self._h, block_id)

    def memoryUsage(self):
        return lib().kvo_cache_memory_usage(self._h)

    def set_free_list(self, ids):
        ids = np.ascontiguousarray(ids, np.uint32)
        return lib().kvo_cache_set_free_list(self._h, _ptr(ids), ids.size)

    def saveToFile(self, path):
        return lib().kvo_cache_save(self._h, os.fsencode(path))

    def loadFromFile(self, path):
        return lib().kvo_cache_load(self._h, os.fsencode(path))

    def cacheBlock(self, block_idx, token_ids, prefix_hash):
        t = np.ascontiguousarray(token_ids, np.uint32)
        lib().kvo_cache_cache_block(self._h, block_idx, _ptr(t), t.size, prefix_hash)

    def findPrefixBlocks(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        return lib().kvo_cache_find_prefix_blocks(self._h, _ptr(t), t.size)

    def reusePrefixBlocks(self, tokens, n_blocks):
        t = np.ascontiguousarray(tokens, np.uint32)
        return lib().kvo_cache_reuse_prefix_blocks(self._h, _ptr(t), t.size, n_blocks)

    def pool(self) -> "_PoolView":
        return _PoolView(lib().kvo_cache_pool(self._h))


class _PoolView(Pool):
    """Borrowed view of a KVCache's pool (not owned, not freed)."""

    def __init__(self, p):  # noqa: D401 - borrowed pointer
        self._view = p
        c = p.contents
        self.n_layers, self.num_blocks, self.block_size = c.n_layers, c.num_blocks, c.block_size
        self.kv_rank, self.rope_dim, self.quantized = c.kv_rank, c.rope_dim, bool(c.quantized)

    @property
    def ref(self):
        return self._view

    def __del__(self):
        pass


# ---------------------------------------------------------------- hashing / generator
def xxh64(data: bytes, seed: int = 0) -> int:
    buf = np.frombuffer(data, np.uint8).copy() if data else np.zeros(1, np.uint8)
    return lib().kvo_xxh64(_ptr(buf), len(data), seed)


def compute_hash(token_ids, prefix_hash: int = NO_HASH) -> int:
    t = np.ascontiguousarray(token_ids, np.uint32)
    return lib().kvo_compute_hash(_ptr(t), t.size, prefix_hash)


def splitmix64(x: int) -> int:
    return lib().kvo_splitmix64(x)


def log_det(s: float) -> float:
    return lib().kvo_log_det(s)


def gen_normal(seed, a, b, c, outlier_p=0.0) -> float:
    return lib().kvo_gen_normal(seed, a, b, c, outlier_p)


def gen_rows(seed, a, b, c, width, outlier_p=0.0, n_threads=None) -> np.ndarray:
    """out[r][i] = gen_normal(seed, a, b[r], c[r]*1024 + i) for i < width."""
    b = np.ascontiguousarray(b, np.uint32)
    c = np.ascontiguousarray(c, np.uint32)
    out = np.zeros((b.size, width), np.float32)
    if n_threads is None:
        n_threads = min(os.cpu_count() or 1, 64)
    lib().kvo_gen_rows(seed, a, b.size, _ptr(b), _ptr(c), width, outlier_p, _ptr(out), n_threads)
    return out
