"""ctypes binding of ``libnifre_b200.so`` (the C ABI declared in include/nifre_b200.h).

The library is built in-tree by ``nifre_b200.build``.  There is no fallback:
if the shared object is missing or a CUDA device is absent, every entry point
raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libnifre_b200.so"

NF_F32, NF_F16, NF_BF16 = 0, 1, 2
NF_STATUS_BAD_BLOCK = 1
NF_STATUS_UNIT_OVERFLOW = 2
NF_STATUS_WAIT_TIMEOUT = 4
NF_STATUS_BAD_SLOT = 8
NF_STATUS_BAD_TILE = 16
NF_STATUS_BAD_SHARED = 32
NF_STATUS_FOREIGN_PARTS = 64

SEQ_FIELDS, PATCH_FIELDS, ITEM_FIELDS, UNIT_FIELDS = 4, 3, 4, 8

_DTYPE_CODE = {torch.float32: NF_F32, torch.float16: NF_F16, torch.bfloat16: NF_BF16}

EXPORTS = ("nf_last_error", "nf_abi_version", "nf_pack_step", "nf_kv_append",
           "nf_attention_workspace", "nf_paged_attention", "nf_paged_attention_noalloc",
           "nf_last_attention_path", "nf_selftest_umma", "nf_prefill_attention", "nf_prefill_tile_rows",
           "nf_cascade_attention", "nf_selftest_wait", "nf_noalloc_scratch_fill", "nf_paged_attention_gather",
           "nf_prefill_attention_gather", "nf_exchange_barrier", "nf_ipc_handle", "nf_ipc_open", "nf_ipc_close", "nf_qkv_append",
           "nf_paged_attention_args", "nf_kv_append_args", "nf_cascade_limits")

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64

MAX_RANKS = 8


class NfGather(ctypes.Structure):
    """struct NfGather of include/nifre_b200.h: a gathered output over the ranks of one node."""
    _fields_ = [("n_ranks", ctypes.c_int32), ("rank", ctypes.c_int32), ("epoch", ctypes.c_int32),
                ("pad", ctypes.c_int32), ("peer_out", ctypes.c_void_p * (MAX_RANKS - 1)),
                ("flags", ctypes.c_void_p * MAX_RANKS), ("epoch_counter", ctypes.c_void_p)]


_G = ctypes.POINTER(NfGather)


class NfAttentionArgs(ctypes.Structure):
    """struct NfAttentionArgs of include/nifre_b200.h (the arguments of nf_paged_attention_gather)."""
    _fields_ = [("out", ctypes.c_void_p), ("out_row_stride", ctypes.c_int64), ("q", ctypes.c_void_p),
                ("q_row_stride", ctypes.c_int64), ("k_pool", ctypes.c_void_p), ("v_pool", ctypes.c_void_p),
                ("dtype", ctypes.c_int32), ("num_q_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("block_size", ctypes.c_int32), ("num_blocks", ctypes.c_int32),
                ("block_tables", ctypes.c_void_p), ("max_blocks_per_seq", ctypes.c_int32),
                ("max_items", ctypes.c_int32), ("max_units", ctypes.c_int32), ("split_tokens", ctypes.c_int32),
                ("items", ctypes.c_void_p), ("units", ctypes.c_void_p), ("counts", ctypes.c_void_p),
                ("scale", ctypes.c_float), ("pad", ctypes.c_int32), ("ws_partials", ctypes.c_void_p),
                ("ws_partial_floats", ctypes.c_int64), ("ws_counters", ctypes.c_void_p),
                ("ws_counter_ints", ctypes.c_int64), ("gather", ctypes.c_void_p), ("status", ctypes.c_void_p)]


class NfAppendArgs(ctypes.Structure):
    """struct NfAppendArgs of include/nifre_b200.h (the arguments of nf_kv_append)."""
    _fields_ = [("k_pool", ctypes.c_void_p), ("v_pool", ctypes.c_void_p), ("pool_rows", ctypes.c_int64),
                ("k_new", ctypes.c_void_p), ("v_new", ctypes.c_void_p), ("k_src_row_stride", ctypes.c_int64),
                ("v_src_row_stride", ctypes.c_int64), ("pool_dtype", ctypes.c_int32), ("src_dtype", ctypes.c_int32),
                ("n_tokens", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("n_seqs", ctypes.c_int32), ("slot_mapping", ctypes.c_void_p), ("src_rows", ctypes.c_void_p),
                ("seqs", ctypes.c_void_p), ("pos_out", ctypes.c_void_p), ("status", ctypes.c_void_p)]

_SIGNATURES = {
    "nf_last_error": ([], ctypes.c_char_p),
    "nf_abi_version": ([], ctypes.c_int),
    "nf_last_attention_path": ([], ctypes.c_int),
    "nf_selftest_umma": ([_P, _P, _P, _I32, _I32, _I32, _P, _P], ctypes.c_int),
    "nf_selftest_wait": ([_I32, _I64, _P, _I32, _P, _P, _P], ctypes.c_int),
    "nf_noalloc_scratch_fill": ([_I32, _P], ctypes.c_int),
    "nf_prefill_tile_rows": ([_I32], ctypes.c_int),
    "nf_prefill_attention": ([_P, _I64, _P, _I64, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                              _P, _I32, _P, _I32, _P, _P, ctypes.c_float, _P, _P], ctypes.c_int),
    "nf_pack_step": ([_P, _I32, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _P, _P,
                      _P, _P, _P, _P, _P, _P, _I32, _I32, _P, _P], ctypes.c_int),
    "nf_cascade_attention": ([_P, _I64, _P, _I64, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I32,
                              _P, _P, _I32, _I32, _P, _I32, _P, _I32, ctypes.c_float, _P, _P], ctypes.c_int),
    "nf_kv_append": ([_P, _P, _I32, _I64, _P, _P, _I32, _I64, _I64, _P, _P, _I32,
                      _I32, _I32, _P, _I32, _P, _P, _P], ctypes.c_int),
    "nf_attention_workspace": ([_I32, _I32, _I32, _I32, _I32, _I32,
                                ctypes.POINTER(_I64), ctypes.POINTER(_I64)], ctypes.c_int),
    "nf_paged_attention": ([_P, _I64, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                            _P, _I32, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float,
                            _P, _I64, _P, _I64, _P, _P], ctypes.c_int),
    "nf_paged_attention_gather": ([_P, _I64, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                   _P, _I32, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float,
                                   _P, _I64, _P, _I64, _G, _P, _P], ctypes.c_int),
    "nf_prefill_attention_gather": ([_P, _I64, _P, _I64, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                     _P, _I32, _P, _I32, _P, _P, ctypes.c_float, _G, _P, _P], ctypes.c_int),
    "nf_exchange_barrier": ([_G, _P, _P], ctypes.c_int),
    "nf_cascade_limits": ([_I32, _I32, _I32, _I32, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_I32)], ctypes.c_int),
    "nf_paged_attention_args": ([_P, _P], ctypes.c_int),
    "nf_kv_append_args": ([_P, _P], ctypes.c_int),
    "nf_qkv_append": ([_P, _I64, _I32, _P, _P, _I32, _I32, _I32, _P, _I64, _P, _P, _I64, _I32, _P, _P, _I32, _P,
                       _P, _P], ctypes.c_int),
    "nf_ipc_handle": ([_P, _P, ctypes.POINTER(_I64)], ctypes.c_int),
    "nf_ipc_open": ([_P, _I64, ctypes.POINTER(_P)], ctypes.c_int),
    "nf_ipc_close": ([_P, _I64], ctypes.c_int),
    "nf_paged_attention_noalloc": ([_P, _I64, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                    _P, _I32, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float,
                                    _P, _P], ctypes.c_int),
}


class NifreError(RuntimeError):
    """A C-ABI call of libnifre_b200 returned an error."""


_lib = None


def load() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NifreError(
                f"{LIB_PATH.name} is missing: build it with `python -m nifre_b200.build` "
                "(the CUDA path has no CPU fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().nf_last_error().decode(errors="replace")
        raise NifreError(f"{what} failed (code {rc}): {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {dtype}") from exc


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """torch's current CUDA stream on ``device`` (raw handle), read without building a Stream object."""
    if _raw_stream is not None:
        idx = device.index if isinstance(device, torch.device) and device.index is not None else \
            torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise NifreError(f"{name} must be a CUDA tensor: nifre_b200 has no CPU path")


def workspace_sizes(max_units: int, max_items: int, hq: int, hkv: int, d: int, dtype: torch.dtype):
    pf, ci = _I64(0), _I64(0)
    check(load().nf_attention_workspace(max_units, max_items, hq, hkv, d, dtype_code(dtype),
                                        ctypes.byref(pf), ctypes.byref(ci)), "nf_attention_workspace")
    return pf.value, ci.value
