"""ctypes binding of libpse.so (the C ABI declared in include/pse.h).

The library is built in-tree (``pse/lib/libpse.so``) by ``pse._build``.  There
is no fallback: importing the engine without the library, or without a CUDA
device, raises.  Every call passes torch's current CUDA stream, so the kernels
are ordered with (and capturable alongside) torch's own work.
"""
from __future__ import annotations

import contextlib
import ctypes
import gc
import os
import threading
from collections import Counter

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libpse.so")

PSE_F32 = 0
PSE_BF16 = 1
STATUS_OOM = 1
STATUS_TABLE_OVERFLOW = 2
STATUS_TRUNCATE_LONG = 4
STATUS_DOUBLE_FREE = 8
STATUS_BAD_BLOCK = 16
STATUS_TIMEOUT = 32
PSE_ESCRATCH = 10003
NOALLOC_SCRATCH_BYTES = 8 << 20

c_p = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_u64 = ctypes.c_uint64
c_sz = ctypes.c_size_t


class BlockState(ctypes.Structure):
    _fields_ = [
        ("block_table", c_p), ("seq_len", c_p), ("nblocks", c_p), ("free_stack", c_p),
        ("free_top", c_p), ("block_free", c_p), ("status", c_p),
        ("num_blocks", c_i32), ("block_size", c_i32), ("max_blocks", c_i32), ("num_slots", c_i32),
    ]


class KVLayer(ctypes.Structure):
    _fields_ = [("k_pool", c_p), ("v_pool", c_p), ("kv_heads", c_i32), ("head_dim", c_i32), ("dtype", c_i32)]


# name -> (argtypes, kernels launched per call)
_PROTOS = {
    "pse_block_init": ([BlockState, c_p], 1),
    "pse_block_alloc_one": ([BlockState, c_p, c_p], 1),
    "pse_block_free_one": ([BlockState, c_p, c_p], 1),
    "pse_kv_reserve": ([BlockState, c_p, c_i32, c_i32, c_p, c_p], 1),
    "pse_kv_reserve_rows": ([BlockState, c_p, c_i32, c_p, c_p, c_p], 1),
    "pse_kv_truncate": ([BlockState, c_p, c_i32, c_p, c_p, c_p, c_p], 1),
    "pse_kv_release": ([BlockState, c_p, c_i32, c_p], 1),
    "pse_kv_append": ([BlockState, KVLayer, c_p, c_p, c_i64, c_i64, c_p, c_p, c_i32, c_i32, c_p], 1),
    "pse_kv_gather": ([BlockState, KVLayer, c_p, c_i32, c_i32, c_p, c_p, c_p], 1),
    "pse_paged_attention": ([BlockState, KVLayer, c_p, c_i64, c_p, c_i64, c_p, c_p, c_i32, c_i32, c_i32,
                             c_f32, c_i32, c_p, c_p, c_sz, c_p], 1),
    "pse_philox_uniforms": ([c_u64, c_p, c_p, c_i32, c_i32, c_p, c_p], 1),
    "pse_sample_tokens": ([c_p, c_i64, c_p, c_i32, c_i32, c_f32, c_p, c_i64, c_i32, c_p, c_i64, c_p, c_i64, c_p], 1),
    "pse_spec_accept": ([c_p, c_i64, c_p, c_p, c_i64, c_i64, c_p, c_i64, c_p, c_p, c_i64, c_i64, c_p, c_p, c_i64,
                         c_i32, c_i32, c_i32, c_f32, c_p, c_p, c_p, c_p], 1),
    "pse_tree_accept": ([c_p, c_i64, c_p, c_p, c_i64, c_p, c_p, c_i64, c_i64, c_i64, c_p, c_i64, c_i64, c_i64, c_p,
                         c_p, c_i64, c_i32, c_i32, c_i32, c_i32, c_f32, c_p, c_p, c_p, c_p, c_p], 1),
    "pse_paged_attention_tree": ([BlockState, KVLayer, c_p, c_i64, c_p, c_i64, c_p, c_p, c_i32, c_i32, c_i32,
                                  c_f32, c_i32, c_p, c_p, c_sz, c_i32, c_i32, c_p], 1),
    "pse_embed_pos": ([c_p, c_p, c_i32, c_i32, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_p, c_p], 1),
    "pse_rope_pos": ([c_p, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_f32, c_i32, c_p], 1),
    "pse_kv_compact": ([BlockState, KVLayer, c_p, c_p, c_p, c_p, c_i32, c_i32, c_p], 1),
    "pse_embed": ([c_p, c_p, c_i32, c_i32, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_p, c_p], 1),
    "pse_norm": ([c_p, c_i64, c_p, c_p, c_i32, c_i32, c_i32, c_f32, c_i32, c_p, c_i64, c_i32, c_p], 1),
    "pse_add_norm": ([c_p, c_i64, c_p, c_i64, c_p, c_i32, c_p, c_p, c_i32, c_i32, c_i32, c_f32, c_i32, c_p, c_i64,
                      c_i32, c_p], 1),
    "pse_epilogue": ([c_i32, c_p, c_i64, c_p, c_p, c_i64, c_p, c_i64, c_i32, c_i32, c_i32, c_p], 1),
    "pse_rope": ([c_p, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_f32, c_i32, c_p], 1),
    "pse_scatter_rows": ([c_p, c_i64, c_p, c_i32, c_i32, c_p, c_i64, c_i32, c_p], 1),
    "pse_attention_force_generic": ([c_i32], 0),
    "pse_accept_select": ([c_i32], 0),
    "pse_launch_overlap": ([c_i32], 0),
    "pse_gemm_pair_tiles": ([c_i32], 0),
    "pse_attention_prefill_select": ([c_i32], 0),
    "pse_gemm_bf16": ([c_p, c_i64, c_p, c_i64, c_p, c_p, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_p], 1),
    "pse_paged_attention_noalloc": ([BlockState, KVLayer, c_p, c_i64, c_p, c_i64, c_p, c_p, c_i32, c_i32, c_i32,
                                     c_f32, c_i32, c_p], 1),
    "pse_sched_commit": ([c_p, c_i32, c_p, c_p, c_i32, c_p, c_p, c_p, c_p, c_p, c_p], 1),
    "pse_step_verify_ids": ([c_p, c_i32, c_p, c_p, c_p, c_i32, c_i32, c_p, c_p, c_p], 1),
    "pse_step_bonus_ids": ([c_p, c_p, c_p, c_p, c_i32, c_i32, c_p, c_p, c_p, c_p], 1),
    "pse_step_finish": ([c_p, c_p, c_p, c_i32, c_p, c_i32, c_p, c_i32, c_p, c_i32, c_p, c_p, c_p, c_p, c_p], 1),
}
_SIZE_PROTOS = {
    "pse_paged_attention_workspace": [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32],
}

_lib = None
_lock = threading.Lock()
launches: Counter = Counter()  # entry point -> calls made from this process


def exported_symbols() -> list[str]:
    return sorted(list(_PROTOS) + list(_SIZE_PROTOS) + ["pse_version", "pse_warmup"])


def load(require_cuda: bool = True):
    """Load libpse.so (once).  Raises if the library is missing, or if
    ``require_cuda`` and no CUDA device is present -- there is no CPU path."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libpse.so not built ({LIB_PATH}); run pse._build.build() -- no CPU fallback exists")
        if require_cuda and not torch.cuda.is_available():
            raise RuntimeError("pse needs a CUDA device (sm_100a); there is no CPU fallback")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (argtypes, _) in _PROTOS.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        for name, argtypes in _SIZE_PROTOS.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = c_sz
        lib.pse_version.restype = ctypes.c_int
        lib.pse_warmup.restype = ctypes.c_int
        _lib = lib
    return _lib


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def call(name: str, *args) -> None:
    lib = _lib if _lib is not None else load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} failed with code {rc}")
    launches[name] += _PROTOS[name][1]


def size_call(name: str, *args) -> int:
    lib = _lib if _lib is not None else load()
    return int(getattr(lib, name)(*args))


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return PSE_F32
    if dtype == torch.bfloat16:
        return PSE_BF16
    raise ValueError(f"unsupported dtype {dtype} (float32 or bfloat16)")


@contextlib.contextmanager
def graph_capture(graph):
    """``torch.cuda.graph(graph)`` with Python's cyclic garbage collector held
    off for the capture.  A collection that runs in the middle of a capture
    frees whatever dead reference cycles hold: CUDA graphs of runners that are
    no longer used, pinned host buffers.  Releasing them makes CUDA calls that
    are not permitted while a stream is capturing, and the capture is then
    invalidated (cudaErrorStreamCaptureInvalidated).  Those cycles are
    collected later, outside any capture."""
    enabled = gc.isenabled()
    gc.disable()
    try:
        with torch.cuda.graph(graph):
            yield
    finally:
        if enabled:
            gc.enable()
