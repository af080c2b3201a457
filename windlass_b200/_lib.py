"""ctypes binding of the C ABI in ``include/wl_attn.h``.

The struct layouts below mirror the header field for field; ``check_abi()``
compares their sizes with the library's own ``sizeof`` values. Loading never
falls back to anything: if ``libwl_attn.so`` is missing or fails to load, the
import raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwl_attn.so")

i32, i64, u32, f32, vp = C.c_int32, C.c_int64, C.c_uint32, C.c_float, C.c_void_p
P_i32 = C.POINTER(C.c_int32)
P_f32 = C.POINTER(C.c_float)

WL_OK, WL_ERR_ARG, WL_ERR_T_EXCEEDS_MAX, WL_ERR_NO_INDICES = 0, 1, 2, 3
WL_ERR_CUDA, WL_ERR_NCCL, WL_ERR_TIMEOUT, WL_ERR_WORKSPACE = 4, 5, 6, 7
WL_ERR_UNSUPPORTED, WL_ERR_DEVICE = 8, 9
WL_MODE_OWNER, WL_MODE_CONSUMER, WL_MODE_DENSE = 0, 1, 2
WL_SEL_CANONICAL = 1


class AttnCfg(C.Structure):
    _fields_ = [("n_heads", i32), ("kv_lora", i32), ("rope_dim", i32), ("idx_heads", i32),
                ("idx_dim", i32), ("index_topk", i32), ("softmax_scale", f32),
                ("idx_qk_scale", f32), ("T_max", i32)]


class LatentCache(C.Structure):
    _fields_ = [("c_kv", vp), ("c_kv_row_stride", i64), ("c_kv_seq_stride", i64),
                ("k_rot", vp), ("k_rot_row_stride", i64), ("k_rot_seq_stride", i64)]


class IndexCache(C.Structure):
    _fields_ = [("keys", vp), ("keys_seq_stride", i64), ("scale", vp), ("scale_seq_stride", i64)]


class Rows(C.Structure):
    _fields_ = [("n_rows", i32), ("rows_per_seq", i32), ("len0", i32), ("len_step", i32)]


class IndexShareC(C.Structure):
    _fields_ = [("idx", vp), ("n_dev", vp), ("stride", i64), ("n", i32), ("producer", u32),
                ("dense", i32)]


class DecodeIO(C.Structure):
    _fields_ = [("batch", i32), ("T", i32), ("latent", LatentCache), ("index", IndexCache),
                ("q_abs", vp), ("q_idx", vp), ("w_idx", vp), ("mode", i32), ("sel_flags", i32),
                ("sel_out", vp), ("sel_n_out", vp), ("sel_in", vp), ("sel_n_in", vp),
                ("sel_n", i32), ("sel_stride", i64), ("index_out", vp), ("index_stride", i64),
                ("ctx", vp), ("lse", vp)]


class PrefillIO(C.Structure):
    _fields_ = [("n_q", i32), ("pos0", i32), ("latent", LatentCache), ("index", IndexCache),
                ("q_abs", vp), ("q_idx", vp), ("w_idx", vp), ("mode", i32), ("sel_flags", i32),
                ("sel_out", vp), ("sel_n_out", vp), ("sel_in", vp), ("sel_n_in", vp),
                ("sel_stride", i64), ("index_out", vp), ("index_stride", i64), ("ctx", vp),
                ("lse", vp)]


class Shard(C.Structure):
    _fields_ = [("t0", i64), ("T_global", i64)]


class CacheAppendIO(C.Structure):
    _fields_ = [("n", i32), ("pos", vp), ("seq", vp), ("cos", vp), ("sin", vp), ("k_raw", vp),
                ("k_norm_w", vp), ("k_norm_b", vp), ("ln_eps", f32), ("index", IndexCache),
                ("kv_raw", vp), ("kv_norm_w", vp), ("rms_eps", f32), ("latent", LatentCache),
                ("n_seq", i32)]


STRUCTS = [AttnCfg, LatentCache, IndexCache, Rows, IndexShareC, DecodeIO, PrefillIO, Shard, CacheAppendIO]

# name -> (restype, argtypes)
SIGNATURES = {
    "wl_strerror": (C.c_char_p, [C.c_int]),
    "wl_abi_version": (i32, []),
    "wl_struct_sizes": (i32, [C.POINTER(i64), i32]),
    "wl_attn_cfg_glm52": (None, [C.POINTER(AttnCfg), i32]),
    "wl_index_share_reset": (None, [C.POINTER(IndexShareC)]),
    "wl_index_share_publish": (None, [C.POINTER(IndexShareC), u32, vp, vp, i64, i32]),
    "wl_index_share_require": (C.c_int, [C.POINTER(IndexShareC), u32]),
    "wl_attn_workspace_bytes": (C.c_size_t, [C.POINTER(AttnCfg), i32, i32]),
    "wl_attn_decode": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(DecodeIO), vp, C.c_size_t, vp]),
    "wl_attn_layer_decode": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(DecodeIO), i32, u32,
                                       C.POINTER(IndexShareC), vp, C.c_size_t, vp]),
    "wl_attn_prefill_workspace_bytes": (C.c_size_t, [C.POINTER(AttnCfg), i32, i32]),
    "wl_attn_prefill": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(PrefillIO), vp, C.c_size_t, vp]),
    "wl_attn_layer_prefill": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(PrefillIO), i32, u32,
                                        C.POINTER(IndexShareC), vp, C.c_size_t, vp]),
    "wl_indexer_scores": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(IndexCache), i32,
                                    C.POINTER(Rows), vp, vp, vp, i64, vp]),
    "wl_indexer_topk": (C.c_int, [vp, i64, C.POINTER(Rows), i32, i32, vp, vp, i64, vp, vp, C.c_size_t, vp]),
    "wl_indexer_topk_workspace_bytes": (C.c_size_t, [i32, i32]),
    "wl_sel_normalize": (C.c_int, [vp, i64, vp, i32, C.POINTER(Rows), i32, vp, i64, vp, vp]),
    "wl_mla_sparse_attn": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(LatentCache), i32,
                                     C.POINTER(Rows), vp, vp, i64, vp, i32, i64, i64, i32, vp,
                                     vp, i32, vp]),
    "wl_lse_merge": (C.c_int, [vp, vp, i32, i32, i64, i64, i64, i64, i32, i32, vp, vp, vp]),
    "wl_comm_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
    "wl_comm_create": (C.c_int, [C.POINTER(C.c_uint8), i32, i32, C.POINTER(vp)]),
    "wl_comm_destroy": (C.c_int, [vp]),
    "wl_comm_p2p": (C.c_int, [vp]),
    "wl_attn_sharded_workspace_bytes": (C.c_size_t, [C.POINTER(AttnCfg), i32, i32, i32]),
    "wl_attn_decode_sharded": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(DecodeIO),
                                         C.POINTER(Shard), vp, vp, C.c_size_t, vp]),
    "wl_device_error": (C.c_int, [i32, C.POINTER(u32)]),
    "wl_attn_decode_noalloc": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(DecodeIO), vp]),
    "wl_cache_append": (C.c_int, [C.POINTER(AttnCfg), C.POINTER(CacheAppendIO), vp]),
    "wl_indexer_query": (C.c_int, [C.POINTER(AttnCfg), i32, vp, i64, vp, vp, i64, i32, vp, vp, vp, vp, vp, vp]),
    "wl_mla_absorb_q": (C.c_int, [C.POINTER(AttnCfg), i32, vp, i64, vp, vp, i64, vp]),
    "wl_mla_project_v": (C.c_int, [C.POINTER(AttnCfg), i32, vp, i64, vp, vp, i64, vp]),
    "wl_diag_set_wait_limit": (C.c_int, [i64]),
    "wl_diag_phase_stamps": (C.c_int, [vp, i32]),
    "wl_diag_phase_count": (i32, []),
    "wl_diag_merge_exchange": (C.c_int, [vp, i64, vp, i32, i32, vp, vp, vp]),
    "wl_diag_xmerge_bytes": (C.c_size_t, [i32]),
    "wl_diag_xmerge": (C.c_int, [i32, i32, i32, vp, vp, vp, C.c_size_t, vp, vp, vp]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (loads on first use; raises if it is absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m windlass_b200.build` "
                "(there is no fallback implementation)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check_abi() -> None:
    """Raise if the ctypes mirrors disagree with the library's struct sizes."""
    L = lib()
    n = L.wl_struct_sizes(None, 0)
    buf = (i64 * n)()
    L.wl_struct_sizes(buf, n)
    if n != len(STRUCTS):
        raise RuntimeError(f"library reports {n} structs, binding has {len(STRUCTS)}")
    for s, size in zip(STRUCTS, buf):
        if C.sizeof(s) != size:
            raise RuntimeError(f"{s.__name__}: ctypes size {C.sizeof(s)} != C size {size}")


class WlError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = lib().wl_strerror(status).decode()
        super().__init__(f"{what}: {msg} (status {status})" if what else f"{msg} (status {status})")


def check(status: int, what: str = "") -> None:
    if status != WL_OK:
        raise WlError(status, what)
