"""Python host interface of the attention substep, shaped like the reference.

The reference's interface for this path is ``run_attention`` with an
``IndexShare`` (src/glm_layer_runner.cuh:485-527) and, on the numpy side,
``indexer_scores`` / ``indexer_topk`` / ``index_drop_mask`` / ``IndexShare``
(tools/ref_glm_chain.py:445-529). This module keeps those names, argument
meanings and error behaviour (a shared layer with nothing published raises
``RuntimeError``) and runs every piece through the C ABI of ``libwl_attn.so``.
PyTorch only supplies device memory and the current CUDA stream.

All tensors are CUDA tensors: bf16 latent cache / queries, uint8 (fp8-e4m3
bit patterns) index keys, fp32 scales, weights and outputs, int32 selections.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import (AttnCfg, DecodeIO, IndexCache, IndexShareC, LatentCache, PrefillIO, Rows,
                   Shard, check, lib)

N_HEADS, KV_LORA, ROPE, IDX_H, IDX_D, INDEX_TOPK = 64, 512, 64, 32, 128, 2048
D_QK = KV_LORA + ROPE


def glm52_cfg(T_max: int, index_topk: int = INDEX_TOPK) -> AttnCfg:
    cfg = AttnCfg()
    lib().wl_attn_cfg_glm52(C.byref(cfg), int(T_max))
    cfg.index_topk = int(index_topk)
    return cfg


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


_ws: dict[int, torch.Tensor] = {}


def workspace(nbytes: int, device: torch.device | None = None) -> torch.Tensor:
    """A per-device caller-owned scratch buffer of at least ``nbytes``."""
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    buf = _ws.get(dev)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=f"cuda:{dev}")
        _ws[dev] = buf
    return buf


@dataclass
class LatentKV:
    """One layer's latent cache: c_kv [S, T, 512] and k_rot [S, T, 64] bf16
    views (S sequences). ``packed(kv)`` splits a [S, T, 576] tensor."""
    c_kv: torch.Tensor
    k_rot: torch.Tensor

    @staticmethod
    def packed(kv: torch.Tensor) -> "LatentKV":
        if kv.dim() == 2:
            kv = kv.unsqueeze(0)
        return LatentKV(kv[..., :KV_LORA], kv[..., KV_LORA:])

    def c(self) -> LatentCache:
        ckv, krt = self.c_kv, self.k_rot
        if ckv.dim() == 2:
            ckv, krt = ckv.unsqueeze(0), krt.unsqueeze(0)
        _need(ckv, torch.bfloat16, "c_kv")
        _need(krt, torch.bfloat16, "k_rot")
        if ckv.stride(-1) != 1 or krt.stride(-1) != 1:
            raise ValueError("latent rows must be contiguous")
        return LatentCache(ckv.data_ptr(), ckv.stride(-2), ckv.stride(0), krt.data_ptr(),
                           krt.stride(-2), krt.stride(0))

    @property
    def T(self) -> int:
        return self.c_kv.shape[-2]


@dataclass
class IndexKeys:
    """An owning layer's indexer key cache: keys [S, T, 128] uint8 (e4m3 bits),
    scale [S, T] fp32."""
    keys: torch.Tensor
    scale: torch.Tensor

    def c(self) -> IndexCache:
        k, s = self.keys, self.scale
        if k.dim() == 2:
            k, s = k.unsqueeze(0), s.unsqueeze(0)
        _need(k, torch.uint8, "index keys")
        _need(s, torch.float32, "index scale")
        if k.stride(-1) != 1 or k.stride(-2) != IDX_D or s.stride(-1) != 1:
            raise ValueError("index keys must be packed [T, 128] rows with contiguous scales")
        return IndexCache(k.data_ptr(), k.stride(0), s.data_ptr(), s.stride(0))


# ---- the individual kernels ------------------------------------------------------------

def indexer_scores(cfg: AttnCfg, keys: IndexKeys, q_idx: torch.Tensor, w_idx: torch.Tensor,
                   T: int, rows: Rows, out: torch.Tensor | None = None) -> torch.Tensor:
    """index[r, t] for t < len(r) (fp32 [n_rows, T]); entries past len(r) are unspecified."""
    _need(q_idx, torch.bfloat16, "q_idx")
    _need(w_idx, torch.float32, "w_idx")
    if out is None:
        out = torch.empty(rows.n_rows, T, dtype=torch.float32, device=q_idx.device)
    check(lib().wl_indexer_scores(C.byref(cfg), C.byref(keys.c()), T, C.byref(rows),
                                  _ptr(q_idx.contiguous()), _ptr(w_idx.contiguous()), _ptr(out),
                                  out.stride(0), _stream()), "wl_indexer_scores")
    return out


def indexer_topk(index: torch.Tensor, k: int, rows: Rows | None = None, T: int | None = None,
                 cand_idx: torch.Tensor | None = None):
    """Exact top-min(k, len) per row, canonical (ascending). Returns (sel, n)."""
    _need(index, torch.float32, "index")
    T = index.shape[1] if T is None else T
    rows = rows or Rows(index.shape[0], 1, T, 0)
    kk = min(k, T)
    sel = torch.full((rows.n_rows, kk), -1, dtype=torch.int32, device=index.device)
    n = torch.empty(rows.n_rows, dtype=torch.int32, device=index.device)
    nbytes = lib().wl_indexer_topk_workspace_bytes(rows.n_rows, T)
    ws = workspace(nbytes, index.device)
    check(lib().wl_indexer_topk(_ptr(index), index.stride(0), C.byref(rows), T, k, _ptr(cand_idx),
                                _ptr(sel), kk, _ptr(n), _ptr(ws), ws.numel(), _stream()), "wl_indexer_topk")
    return sel, n


def sel_normalize(sel_in: torch.Tensor, T: int, n_in: torch.Tensor | None = None,
                  rows: Rows | None = None):
    """Canonical list of the keys an arbitrary list keeps (the mask semantics)."""
    _need(sel_in, torch.int32, "sel_in")
    rows = rows or Rows(sel_in.shape[0], 1, T, 0)
    out = torch.full((rows.n_rows, T), -1, dtype=torch.int32, device=sel_in.device)
    n = torch.empty(rows.n_rows, dtype=torch.int32, device=sel_in.device)
    check(lib().wl_sel_normalize(_ptr(sel_in), sel_in.stride(0), _ptr(n_in), sel_in.shape[1],
                                 C.byref(rows), T, _ptr(out), out.stride(0), _ptr(n), _stream()),
          "wl_sel_normalize")
    return out, n


def mla_sparse_attn(cfg: AttnCfg, kv: LatentKV, q_abs: torch.Tensor, rows: Rows,
                    sel: torch.Tensor | None = None, sel_n: torch.Tensor | int | None = None,
                    win: tuple[int, int] | None = None, split_keys: int = 0,
                    max_splits: int = 1):
    """Partials (o [n_rows, max_splits, 64, 512], lse [n_rows, max_splits, 64])."""
    _need(q_abs, torch.bfloat16, "q_abs")
    T = kv.T
    lo, hi = win if win is not None else (0, T)
    o = torch.empty(rows.n_rows, max_splits, N_HEADS, KV_LORA, dtype=torch.float32, device=q_abs.device)
    lse = torch.empty(rows.n_rows, max_splits, N_HEADS, dtype=torch.float32, device=q_abs.device)
    n_dev = sel_n if isinstance(sel_n, torch.Tensor) else None
    n_host = int(sel_n) if isinstance(sel_n, int) else (sel.shape[1] if sel is not None else 0)
    check(lib().wl_mla_sparse_attn(C.byref(cfg), C.byref(kv.c()), T, C.byref(rows),
                                   _ptr(q_abs.contiguous()), _ptr(sel),
                                   sel.stride(0) if sel is not None else 0, _ptr(n_dev), n_host,
                                   lo, hi, split_keys, _ptr(o), _ptr(lse), max_splits, _stream()),
          "wl_mla_sparse_attn")
    return o, lse


def lse_merge(o_part: torch.Tensor, lse_part: torch.Tensor):
    """Merge [R, S, H, D] partials into (ctx [R, H, D], lse [R, H])."""
    R, S, H, D = o_part.shape
    ctx = torch.empty(R, H, D, dtype=torch.float32, device=o_part.device)
    lse = torch.empty(R, H, dtype=torch.float32, device=o_part.device)
    check(lib().wl_lse_merge(_ptr(o_part), _ptr(lse_part), R, S, S * H * D, H * D, S * H, H, H, D,
                             _ptr(ctx), _ptr(lse), _stream()), "wl_lse_merge")
    return ctx, lse


# ---- the indexer's query side ------------------------------------------------------------------

def indexer_query(cfg: AttnCfg, q_resid: torch.Tensor, wq_b: torch.Tensor, x: torch.Tensor,
                  weights_proj: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """(q_idx bf16 [n, 32, 128], w_idx fp32 [n, 32]) from q_resid fp32 [n, 2048],
    wq_b bf16 [4096, 2048], x fp32 [n, hidden], weights_proj fp32 [32, hidden] and
    the rows' RoPE tables [n, 32] (``wl_indexer_query``; the query half of
    launch_indexer_query, src/glm_kernels.cuh:469-472; numpy indexer_scores'
    q and w, tools/ref_glm_chain.py:482-501)."""
    for t, dt, nm in ((q_resid, torch.float32, "q_resid"), (wq_b, torch.bfloat16, "wq_b"),
                      (x, torch.float32, "x"), (weights_proj, torch.float32, "weights_proj"),
                      (cos, torch.float32, "cos"), (sin, torch.float32, "sin")):
        _need(t, dt, nm)
    q_resid, x = q_resid.contiguous(), x.contiguous()
    wq_b, weights_proj, cos, sin = wq_b.contiguous(), weights_proj.contiguous(), cos.contiguous(), sin.contiguous()
    n, hidden = x.shape
    q_idx = torch.empty(n, IDX_H, IDX_D, dtype=torch.bfloat16, device=x.device)
    w_idx = torch.empty(n, IDX_H, dtype=torch.float32, device=x.device)
    check(lib().wl_indexer_query(C.byref(cfg), n, _ptr(q_resid), q_resid.stride(0), _ptr(wq_b), _ptr(x),
                                 x.stride(0), hidden, _ptr(weights_proj), _ptr(cos), _ptr(sin), _ptr(q_idx),
                                 _ptr(w_idx), _stream()), "wl_indexer_query")
    return q_idx, w_idx


# ---- the absorption around the attention ------------------------------------------------------

def mla_absorb_q(cfg: AttnCfg, q: torch.Tensor, kv_b: torch.Tensor) -> torch.Tensor:
    """q fp32 [n, 64, 256] (qk_nope | roped qk_rope), kv_b bf16 [64 * 448, 512]
    -> the attention's absorbed query, bf16 [n, 64, 576] (``wl_mla_absorb_q``;
    mla_absorb_q, src/glm_layer_runner.cuh:196-215)."""
    _need(q, torch.float32, "q")
    _need(kv_b, torch.bfloat16, "kv_b")
    q, kv_b = q.reshape(-1, N_HEADS * 256).contiguous(), kv_b.contiguous()
    out = torch.empty(q.shape[0], N_HEADS, D_QK, dtype=torch.bfloat16, device=q.device)
    check(lib().wl_mla_absorb_q(C.byref(cfg), q.shape[0], _ptr(q), q.stride(0), _ptr(kv_b), _ptr(out),
                                N_HEADS * D_QK, _stream()), "wl_mla_absorb_q")
    return out


def mla_project_v(cfg: AttnCfg, ctx: torch.Tensor, kv_b: torch.Tensor) -> torch.Tensor:
    """ctx fp32 [n, 64, 512] -> fp32 [n, 64, 256] through W_UV (``wl_mla_project_v``;
    mla_project_v, src/glm_layer_runner.cuh:217-234)."""
    _need(ctx, torch.float32, "ctx")
    _need(kv_b, torch.bfloat16, "kv_b")
    ctx, kv_b = ctx.reshape(-1, N_HEADS * KV_LORA).contiguous(), kv_b.contiguous()
    out = torch.empty(ctx.shape[0], N_HEADS, 256, dtype=torch.float32, device=ctx.device)
    check(lib().wl_mla_project_v(C.byref(cfg), ctx.shape[0], _ptr(ctx), ctx.stride(0), _ptr(kv_b), _ptr(out),
                                 N_HEADS * 256, _stream()), "wl_mla_project_v")
    return out


# ---- the cache write path ---------------------------------------------------------------------

def cache_append(cfg: AttnCfg, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
                 keys: IndexKeys | None = None, k_raw: torch.Tensor | None = None,
                 k_norm_w: torch.Tensor | None = None, k_norm_b: torch.Tensor | None = None,
                 ln_eps: float = 1e-6, kv: LatentKV | None = None, kv_raw: torch.Tensor | None = None,
                 kv_norm_w: torch.Tensor | None = None, rms_eps: float = 1e-6,
                 seq: torch.Tensor | None = None) -> None:
    """Write n tokens into the caches (``wl_cache_append``): the reference's
    ``launch_indexer_key`` (src/glm_kernels.cuh:432-448; numpy
    ``indexer_keys``, tools/ref_glm_chain.py:465-480) into ``keys`` from
    ``k_raw`` = wk(x) [n, 128] fp32, and the latent row write of
    ``run_attention`` (src/glm_layer_runner.cuh:544-570) into ``kv`` from
    ``kv_raw`` = kv_a_proj_with_mqa(x) [n, 576] fp32. ``pos`` [n] int32 rows,
    ``seq`` [n] int32 sequences (None: 0), ``cos``/``sin`` [n, 32] fp32 the
    tokens' RoPE table rows; norm weights/bias bf16."""
    _need(pos, torch.int32, "pos")
    _need(cos, torch.float32, "cos")
    _need(sin, torch.float32, "sin")
    n = pos.numel()
    io = _lib.CacheAppendIO()
    io.n = n
    hold = [pos.contiguous(), cos.contiguous(), sin.contiguous()]
    io.pos, io.cos, io.sin = (t.data_ptr() for t in hold)
    if seq is not None:
        _need(seq, torch.int32, "seq")
        hold.append(seq.contiguous())
        io.seq = hold[-1].data_ptr()
    if k_raw is not None:
        if keys is None or k_norm_w is None or k_norm_b is None:
            raise ValueError("k_raw needs keys, k_norm_w and k_norm_b")
        _need(k_raw, torch.float32, "k_raw")
        _need(k_norm_w, torch.bfloat16, "k_norm_w")
        _need(k_norm_b, torch.bfloat16, "k_norm_b")
        hold += [k_raw.contiguous(), k_norm_w.contiguous(), k_norm_b.contiguous()]
        io.k_raw, io.k_norm_w, io.k_norm_b = (t.data_ptr() for t in hold[-3:])
        io.ln_eps = ln_eps
        io.index = keys.c()
    if kv_raw is not None:
        if kv is None or kv_norm_w is None:
            raise ValueError("kv_raw needs kv and kv_norm_w")
        _need(kv_raw, torch.float32, "kv_raw")
        _need(kv_norm_w, torch.bfloat16, "kv_norm_w")
        hold += [kv_raw.contiguous(), kv_norm_w.contiguous()]
        io.kv_raw, io.kv_norm_w = (t.data_ptr() for t in hold[-2:])
        io.rms_eps = rms_eps
        io.latent = kv.c()
    # sequences the given caches hold: the library skips (and flags) any seq[i] outside them
    counts = []
    if k_raw is not None:
        counts.append(keys.keys.shape[0] if keys.keys.dim() == 3 else 1)
    if kv_raw is not None:
        counts.append(kv.c_kv.shape[0] if kv.c_kv.dim() == 3 else 1)
    io.n_seq = min(counts) if seq is not None else 1
    check(lib().wl_cache_append(C.byref(cfg), C.byref(io), _stream()), "wl_cache_append")


# ---- the substep ----------------------------------------------------------------------------

def decode_io(cfg: AttnCfg, kv: LatentKV, q_abs: torch.Tensor, *, keys: IndexKeys | None = None,
              q_idx: torch.Tensor | None = None, w_idx: torch.Tensor | None = None,
              mode: int = _lib.WL_MODE_OWNER, sel_in: torch.Tensor | None = None,
              sel_n_in: torch.Tensor | None = None, sel_n: int | None = None,
              canonical: bool = False, sel_out: torch.Tensor | None = None,
              sel_n_out: torch.Tensor | None = None, index_out: torch.Tensor | None = None,
              ctx: torch.Tensor | None = None, lse: torch.Tensor | None = None) -> tuple[DecodeIO, dict]:
    """Fill a DecodeIO; returns it with the tensors it points to (keep them alive)."""
    B = q_abs.shape[0]
    T = kv.T
    dev = q_abs.device
    kk = min(cfg.index_topk, T)
    if ctx is None:
        ctx = torch.empty(B, N_HEADS, KV_LORA, dtype=torch.float32, device=dev)
    if lse is None:
        lse = torch.empty(B, N_HEADS, dtype=torch.float32, device=dev)
    if mode == _lib.WL_MODE_OWNER:
        if sel_out is None:
            sel_out = torch.empty(B, kk, dtype=torch.int32, device=dev)
        if sel_n_out is None:
            sel_n_out = torch.empty(B, dtype=torch.int32, device=dev)
    io = DecodeIO()
    io.batch, io.T = B, T
    io.latent = kv.c()
    if keys is not None:
        io.index = keys.c()
    io.q_abs = _ptr(q_abs)
    io.q_idx = _ptr(q_idx)
    io.w_idx = _ptr(w_idx)
    io.mode = mode
    io.sel_flags = _lib.WL_SEL_CANONICAL if canonical else 0
    io.sel_out = _ptr(sel_out)
    io.sel_n_out = _ptr(sel_n_out)
    io.sel_in = _ptr(sel_in)
    io.sel_n_in = _ptr(sel_n_in)
    io.sel_n = int(sel_n if sel_n is not None else (sel_in.shape[1] if sel_in is not None else 0))
    if sel_out is not None:
        io.sel_stride = sel_out.stride(0)
    elif sel_in is not None:
        io.sel_stride = sel_in.stride(0)
    io.index_out = _ptr(index_out)
    io.index_stride = index_out.stride(0) if index_out is not None else 0
    io.ctx = _ptr(ctx)
    io.lse = _ptr(lse)
    keep = dict(ctx=ctx, lse=lse, sel=sel_out, sel_n=sel_n_out, sel_out=sel_out, sel_n_out=sel_n_out,
                index_out=index_out,
                q_abs=q_abs, q_idx=q_idx, w_idx=w_idx, sel_in=sel_in, sel_n_in=sel_n_in, kv=kv,
                keys=keys)
    return io, keep


def attn_decode(cfg: AttnCfg, kv: LatentKV, q_abs: torch.Tensor, **kw) -> dict:
    """One decode token per sequence through ``wl_attn_decode``.

    Returns the output tensors: ctx [B,64,512], lse [B,64] and, for an owner,
    sel [B,k'] (canonical) with counts sel_n [B]."""
    io, keep = decode_io(cfg, kv, q_abs, **kw)
    nbytes = lib().wl_attn_workspace_bytes(C.byref(cfg), io.T, io.batch)
    ws = workspace(nbytes, q_abs.device)
    check(lib().wl_attn_decode(C.byref(cfg), C.byref(io), _ptr(ws), ws.numel(), _stream()),
          "wl_attn_decode")
    return keep


class IndexShare:
    """``prev_topk_indices`` threaded through the layer loop
    (glm_layer_runner.cuh:485-517; tools/ref_glm_chain.py:445-462).

    Owners publish their raw selection; shared layers read it unchanged (no
    consume-and-clear); a shared layer with nothing published raises
    ``RuntimeError``. ``dense`` is the standalone-layer test mode."""

    def __init__(self, dense: bool = False):
        self.c = IndexShareC()
        self.c.dense = int(dense)
        lib().wl_index_share_reset(C.byref(self.c))
        self._keep: tuple = ()

    def reset(self) -> None:
        lib().wl_index_share_reset(C.byref(self.c))
        self._keep = ()

    @property
    def producer(self) -> int | None:
        p = self.c.producer
        return None if p == 0xFFFFFFFF else p

    @property
    def dense(self) -> bool:
        return bool(self.c.dense)

    def publish(self, layer: int, idx: torch.Tensor, n: torch.Tensor) -> None:
        lib().wl_index_share_publish(C.byref(self.c), layer, _ptr(idx), _ptr(n), idx.stride(0),
                                     idx.shape[1])
        self._keep = (idx, n)

    @property
    def indices(self):
        return self._keep[0] if self._keep else None

    def require(self, layer: int) -> None:
        st = lib().wl_index_share_require(C.byref(self.c), layer)
        if st == _lib.WL_ERR_NO_INDICES:
            raise RuntimeError(
                f'layer {layer} is "shared" and has no published indices; its group leader '
                "must run first (IndexShare is empty)")
        check(st, "IndexShare.require")


def run_attention(cfg: AttnCfg, layer: int, owner: bool, share: IndexShare, kv: LatentKV,
                  q_abs: torch.Tensor, keys: IndexKeys | None = None,
                  q_idx: torch.Tensor | None = None, w_idx: torch.Tensor | None = None) -> dict:
    """The hot block of run_attention (glm_layer_runner.cuh:582-644) for one
    decode token per sequence, through ``wl_attn_layer_decode``."""
    B, T = q_abs.shape[0], kv.T
    kk = min(cfg.index_topk, T)
    dev = q_abs.device
    sel_out = sel_n_out = None
    if owner:
        sel_out = torch.empty(B, kk, dtype=torch.int32, device=dev)
        sel_n_out = torch.empty(B, dtype=torch.int32, device=dev)
    io, keep = decode_io(cfg, kv, q_abs, keys=keys, q_idx=q_idx, w_idx=w_idx,
                         mode=_lib.WL_MODE_OWNER if owner else _lib.WL_MODE_CONSUMER,
                         sel_out=sel_out, sel_n_out=sel_n_out)
    nbytes = lib().wl_attn_workspace_bytes(C.byref(cfg), T, B)
    ws = workspace(nbytes, dev)
    st = lib().wl_attn_layer_decode(C.byref(cfg), C.byref(io), int(owner), layer, C.byref(share.c),
                                    _ptr(ws), ws.numel(), _stream())
    if st == _lib.WL_ERR_NO_INDICES:
        share.require(layer)  # raises with the reference's message
    check(st, "wl_attn_layer_decode")
    if owner:
        share._keep = (sel_out, sel_n_out)
    return keep


def attn_prefill(cfg: AttnCfg, kv: LatentKV, q_abs: torch.Tensor, pos0: int, *,
                 keys: IndexKeys | None = None, q_idx: torch.Tensor | None = None,
                 w_idx: torch.Tensor | None = None, mode: int = _lib.WL_MODE_OWNER,
                 sel_in: torch.Tensor | None = None, sel_n_in: torch.Tensor | None = None,
                 canonical: bool = False, index_out: torch.Tensor | None = None) -> dict:
    """Chunked prefill of n_q rows after a pos0-token prefix (row i causal over
    keys [0, pos0+i]) through ``wl_attn_prefill``."""
    n_q = q_abs.shape[0]
    T = pos0 + n_q
    dev = q_abs.device
    kk = min(cfg.index_topk, T)
    ctx = torch.empty(n_q, N_HEADS, KV_LORA, dtype=torch.float32, device=dev)
    lse = torch.empty(n_q, N_HEADS, dtype=torch.float32, device=dev)
    sel_out = sel_n_out = None
    if mode == _lib.WL_MODE_OWNER:
        sel_out = torch.full((n_q, kk), -1, dtype=torch.int32, device=dev)
        sel_n_out = torch.empty(n_q, dtype=torch.int32, device=dev)
    io = PrefillIO()
    io.n_q, io.pos0 = n_q, pos0
    io.latent = kv.c()
    if keys is not None:
        io.index = keys.c()
    io.q_abs, io.q_idx, io.w_idx = _ptr(q_abs), _ptr(q_idx), _ptr(w_idx)
    io.mode = mode
    io.sel_flags = _lib.WL_SEL_CANONICAL if canonical else 0
    io.sel_out, io.sel_n_out = _ptr(sel_out), _ptr(sel_n_out)
    io.sel_in, io.sel_n_in = _ptr(sel_in), _ptr(sel_n_in)
    io.sel_stride = sel_out.stride(0) if sel_out is not None else (sel_in.stride(0) if sel_in is not None else 0)
    io.index_out = _ptr(index_out)
    io.index_stride = index_out.stride(0) if index_out is not None else 0
    io.ctx, io.lse = _ptr(ctx), _ptr(lse)
    nbytes = lib().wl_attn_prefill_workspace_bytes(C.byref(cfg), n_q, T)
    ws = workspace(nbytes, dev)
    check(lib().wl_attn_prefill(C.byref(cfg), C.byref(io), _ptr(ws), ws.numel(), _stream()),
          "wl_attn_prefill")
    return dict(ctx=ctx, lse=lse, sel=sel_out, sel_n=sel_n_out)


def run_prefill_attention(cfg: AttnCfg, layer: int, owner: bool, share: IndexShare, kv: LatentKV,
                          q_abs: torch.Tensor, pos0: int, keys: IndexKeys | None = None,
                          q_idx: torch.Tensor | None = None, w_idx: torch.Tensor | None = None) -> dict:
    """The attention substep of one layer of run_prefill_layer_major
    (glm_layer_runner.cuh:954-983) for a chunk of n_q rows after pos0, through
    ``wl_attn_layer_prefill``: owners publish every row's selection, shared
    layers attend each row over its own published row."""
    n_q = q_abs.shape[0]
    T = pos0 + n_q
    kk = min(cfg.index_topk, T)
    dev = q_abs.device
    ctx = torch.empty(n_q, N_HEADS, KV_LORA, dtype=torch.float32, device=dev)
    sel_out = sel_n_out = None
    if owner:
        sel_out = torch.full((n_q, kk), -1, dtype=torch.int32, device=dev)
        sel_n_out = torch.empty(n_q, dtype=torch.int32, device=dev)
    io = PrefillIO()
    io.n_q, io.pos0 = n_q, pos0
    io.latent = kv.c()
    if keys is not None:
        io.index = keys.c()
    io.q_abs, io.q_idx, io.w_idx = _ptr(q_abs), _ptr(q_idx), _ptr(w_idx)
    io.sel_out, io.sel_n_out = _ptr(sel_out), _ptr(sel_n_out)
    io.sel_stride = sel_out.stride(0) if sel_out is not None else 0
    io.ctx = _ptr(ctx)
    nbytes = lib().wl_attn_prefill_workspace_bytes(C.byref(cfg), n_q, T)
    ws = workspace(nbytes, dev)
    st = lib().wl_attn_layer_prefill(C.byref(cfg), C.byref(io), int(owner), layer, C.byref(share.c),
                                     _ptr(ws), ws.numel(), _stream())
    if st == _lib.WL_ERR_NO_INDICES:
        share.require(layer)  # raises with the reference's message
    check(st, "wl_attn_layer_prefill")
    if owner:
        share._keep = (sel_out, sel_n_out)
    return dict(ctx=ctx, sel=sel_out, sel_n=sel_n_out)


def device_error(clear: bool = True) -> tuple[int, int]:
    """(status, raw word) of the library's device-side error word."""
    w = C.c_uint32(0)
    st = lib().wl_device_error(int(clear), C.byref(w))
    return st, w.value


# ---- KV-sequence sharding ---------------------------------------------------------------------

class Comm:
    """The library's communicator (NVLink peer exchange, else NCCL), bootstrapped
    through torch.distributed. Creation and close() are collective."""

    def __init__(self, rank: int, world: int, group=None):
        import torch.distributed as dist
        uid = (C.c_uint8 * 128)()
        if rank == 0:
            check(lib().wl_comm_unique_id(uid), "wl_comm_unique_id")
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0, group=group)
        uid = (C.c_uint8 * 128).from_buffer_copy(obj[0])
        h = C.c_void_p()
        check(lib().wl_comm_create(uid, world, rank, C.byref(h)), "wl_comm_create")
        self.h, self.rank, self.world = h, rank, world

    @property
    def p2p(self) -> bool:
        """True when the exchanges run over NVLink peer memory."""
        return bool(lib().wl_comm_p2p(self.h))

    def close(self) -> None:
        if self.h:
            lib().wl_comm_destroy(self.h)
            self.h = None


def attn_decode_sharded(cfg: AttnCfg, comm: Comm, t0: int, T_global: int, kv: LatentKV,
                        q_abs: torch.Tensor, **kw) -> dict:
    """Decode with this rank holding keys [t0, t0 + kv.T) of every cache."""
    B = q_abs.shape[0]
    dev = q_abs.device
    kg = min(cfg.index_topk, T_global)
    if kw.get("mode", _lib.WL_MODE_OWNER) == _lib.WL_MODE_OWNER:
        kw.setdefault("sel_out", torch.full((B, kg), -1, dtype=torch.int32, device=dev))
        kw.setdefault("sel_n_out", torch.empty(B, dtype=torch.int32, device=dev))
    io, keep = decode_io(cfg, kv, q_abs, **kw)
    shard = Shard(t0, T_global)
    nbytes = lib().wl_attn_sharded_workspace_bytes(C.byref(cfg), kv.T, B, comm.world)
    ws = workspace(nbytes, dev)
    check(lib().wl_attn_decode_sharded(C.byref(cfg), C.byref(io), C.byref(shard), comm.h, _ptr(ws),
                                       ws.numel(), _stream()), "wl_attn_decode_sharded")
    return keep
