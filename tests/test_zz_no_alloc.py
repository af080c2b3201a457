"""wl_attn_decode_noalloc: decode attention for callers that cannot allocate
device memory (code where cudaMalloc is off limits, or a host runtime that
owns every allocation and only lends input and output buffers). It must give
the same results as wl_attn_decode, which takes a caller workspace, on
consecutive calls that reuse its fixed internal scratch.

This file is collected last on purpose (the name sorts after the others), so
that a run stopping at its first failure has already run everything else.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import attn_ref as o
from windlass_b200 import _lib
from windlass_b200 import attn as A

pytestmark = pytest.mark.gpu

ULP_TOL = 2.0  # the GPU tests' attention tolerance: 2 bf16 ulp of the output scale


def _gpu(inps):
    st = lambda k: np.stack([i[k] for i in inps])  # noqa: E731
    d = lambda x, t: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(t)  # noqa: E731
    kv = A.LatentKV(d(st("c_kv"), torch.bfloat16), d(st("k_rot"), torch.bfloat16))
    return kv, d(st("q_abs"), torch.bfloat16)


def _noalloc(cfg, kv, q_abs, **kw):
    io, keep = A.decode_io(cfg, kv, q_abs, **kw)
    st = _lib.lib().wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "wl_attn_decode_noalloc")
    torch.cuda.synchronize()
    return keep


def _same(ref, got):
    r, g = ref["ctx"].cpu().numpy(), got["ctx"].cpu().numpy()
    for b in range(r.shape[0]):
        assert o.bf16_ulp_error(r[b], g[b]) <= ULP_TOL
    assert torch.allclose(ref["lse"], got["lse"], atol=1e-3, rtol=0)


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    A.device_error(clear=True)
    # call 1: three sequences consuming a canonical selection of 2048 of 5000 keys
    T = 5000
    inps = [o.make_inputs(T, 1, seq=s) for s in range(3)]
    kv, q_abs = _gpu(inps)
    cfg = A.glm52_cfg(T)
    rng = np.random.default_rng(5)
    sel = np.stack([np.sort(rng.choice(T, 2048, replace=False)) for _ in range(3)]).astype(np.int32)
    sel_t = torch.from_numpy(sel).cuda()
    kw = dict(mode=_lib.WL_MODE_CONSUMER, sel_in=sel_t, canonical=True)
    ref = A.attn_decode(cfg, kv, q_abs, **kw)
    got = _noalloc(cfg, kv, q_abs, **kw)
    _same(ref, got)
    # call 2, straight after, on the same scratch: two other sequences, dense
    T2 = 1500
    inps2 = [o.make_inputs(T2, 0, seq=s) for s in range(2)]
    kv2, q2 = _gpu(inps2)
    cfg2 = A.glm52_cfg(T2)
    ref2 = A.attn_decode(cfg2, kv2, q2, mode=_lib.WL_MODE_DENSE)
    got2 = _noalloc(cfg2, kv2, q2, mode=_lib.WL_MODE_DENSE)
    _same(ref2, got2)
    # and against the oracle, to be sure both agree with the reference algorithm
    rc, _ = o.mla_absorbed(inps2[1]["q_abs"], inps2[1]["c_kv"], inps2[1]["k_rot"], None, 1 / 16)
    assert o.bf16_ulp_error(rc, got2["ctx"].cpu().numpy()[1]) <= ULP_TOL
    st, word = A.device_error(clear=True)
    assert st == _lib.WL_OK, f"device error word 0x{word:08x}"


def test_noalloc_rejects_batches_beyond_its_fixed_scratch():
    T = 256
    inps = [o.make_inputs(T, 0, seq=s) for s in range(5)]
    kv, q_abs = _gpu(inps)
    cfg = A.glm52_cfg(T)
    io, keep = A.decode_io(cfg, kv, q_abs, mode=_lib.WL_MODE_DENSE)
    st = _lib.lib().wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.WL_ERR_WORKSPACE


def test_noalloc_without_lse_and_with_device_counts():
    """Two more shapes of a call: no lse output (the attention's merge then
    writes its lse into the fixed scratch) and a consumer whose per-sequence
    counts come from device memory (ragged lists of one stride)."""
    A.device_error(clear=True)
    T = 3000
    inps = [o.make_inputs(T, 1, seq=10 + s) for s in range(4)]
    kv, q_abs = _gpu(inps)
    cfg = A.glm52_cfg(T)
    rng = np.random.default_rng(17)
    counts = [2048, 700, 1, 1999]
    sel = np.full((4, 2048), -1, np.int32)
    for b, n in enumerate(counts):
        sel[b, :n] = np.sort(rng.choice(T, n, replace=False))
    sel_t = torch.from_numpy(sel).cuda()
    n_t = torch.tensor(counts, dtype=torch.int32, device="cuda")
    kw = dict(mode=_lib.WL_MODE_CONSUMER, sel_in=sel_t, sel_n_in=n_t, canonical=True)
    ref = A.attn_decode(cfg, kv, q_abs, **kw)
    got = _noalloc(cfg, kv, q_abs, **kw)
    _same(ref, got)
    # the same call with io.lse = NULL: ctx is unchanged
    io, keep = A.decode_io(cfg, kv, q_abs, **kw)
    io.lse = None
    _lib.check(_lib.lib().wl_attn_decode_noalloc(C.byref(cfg), C.byref(io), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(keep["ctx"], got["ctx"])
    for b, n in enumerate(counts):
        rc, _ = o.mla_sparse(inps[b]["q_abs"], inps[b]["c_kv"], inps[b]["k_rot"], sel[b, :n], 1 / 16)
        assert o.bf16_ulp_error(rc, keep["ctx"].cpu().numpy()[b]) <= ULP_TOL
    st, word = A.device_error(clear=True)
    assert st == _lib.WL_OK, f"device error word 0x{word:08x}"
