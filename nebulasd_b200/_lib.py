"""ctypes binding of ``libnebula_b200.so`` (the C ABI of ``include/nebula_b200.h``).

The library is built in-tree by ``python -m nebulasd_b200.build``.  There is no
fallback: if the shared object is missing or does not load, importing any op
module raises, so a GPU run can never silently take another path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PATH = Path(os.environ.get("NEB_LIBRARY", Path(__file__).resolve().parent / "libnebula_b200.so"))

if not _PATH.exists():
    raise ImportError(f"{_PATH} is missing: build it with `python -m nebulasd_b200.build`")

lib = ctypes.CDLL(str(_PATH))

_vp, _i32, _i64, _f32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
_u32p = ctypes.POINTER(ctypes.c_uint32)

_ATTN = [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i32,
         _f32, _vp, _vp, _sz, _vp]

SIGNATURES = {
    "neb_version": ([], ctypes.c_int),
    "neb_last_error": ([], ctypes.c_char_p),
    "neb_attention_workspace_bytes": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int], _sz),
    "neb_attention_max_rows": ([ctypes.c_int], ctypes.c_int),
    "neb_paged_attention_decode": (_ATTN, ctypes.c_int),
    "neb_paged_attention_verify": (_ATTN, ctypes.c_int),
    "neb_paged_attention_verify_long": (_ATTN, ctypes.c_int),
    "neb_paged_attention_decode_noalloc": (_ATTN[:18] + [_vp], ctypes.c_int),
    "neb_paged_attention_noalloc_status": ([_u32p, _vp], ctypes.c_int),
    "neb_workspace_status": ([_vp, _u32p, _vp], ctypes.c_int),
    "neb_qk_norm_rope_store": ([_vp, _vp, _vp, _vp, _vp, _f32, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp,
                                _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i32, _vp,
                                _vp], ctypes.c_int),
    "neb_store_kvcache": ([_vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32,
                           _i32, _i32, _i64, _i32, _i32, _vp, _vp], ctypes.c_int),
    "neb_rmsnorm_inplace": ([_vp, _vp, _i64, _i32, _f32, _vp], ctypes.c_int),
    "neb_rotary_inplace": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp], ctypes.c_int),
    "neb_hostkv_copy": ([ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _vp, _i32, _i32, _vp], ctypes.c_int),
    "neb_kv_peer_copy": ([_vp, _vp, _vp, _vp, _i64, _vp, _i32, _i32, _vp], ctypes.c_int),
    "neb_host_device_pointer": ([_vp, ctypes.POINTER(_vp)], ctypes.c_int),
    "neb_enable_peer_access": ([ctypes.c_int], ctypes.c_int),
    "neb_greedy_accept_workspace_bytes": ([_i32], _sz),
    "neb_greedy_accept": ([_vp, _i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                           _sz, _vp], ctypes.c_int),
    "neb_prefill_attention_workspace_bytes": ([_i64, _i32, _i32, _i32], _sz),
    "neb_prefill_attention": ([_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i32, _i64, _i32, _i32, _i32, _i32, ctypes.c_float,
                               _vp, _i64, _vp, _sz, _vp], ctypes.c_int),
}

for _name, (_args, _res) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _res

NEB_ERR_INVALID, NEB_ERR_UNSUPPORTED, NEB_ERR_CUDA, NEB_ERR_WORKSPACE, NEB_ERR_DEVICE = 1, 2, 3, 4, 5
NEB_ATTN_DECODE = 0
NEB_ATTN_VERIFY = 1
NEB_ATTN_VERIFY_LONG = 2


class NebError(RuntimeError):
    """A C entry point returned a non-zero status."""


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib.neb_last_error().decode(errors="replace")
        raise NebError(f"{what} failed (status {rc}): {msg}")


def ptr(t) -> int | None:
    """Device/host address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
