"""Failure detection on one GPU without a GPU fault: a bounded device-side wait
runs out, the kernel records WL_ERR_TIMEOUT in the device error word and
returns, and the context stays usable.

The reference aborts the process on any CUDA error (GLM_CUDA_OK,
src/glm_loader.cuh:24-26). Here every wait is bounded (mbarrier waits and the
peer-exchange word waits). The consumer of the sharded decode's (o, lse)
exchange is driven through a test hook over a caller-made region whose words
carry an epoch that never arrives; the wait limit is shortened to ~1 ms so the
timeout comes quickly. Nothing here hangs or faults: the waits end by
themselves and the kernels return.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import attn_ref as o
from windlass_b200 import _lib
from windlass_b200 import attn as A

pytestmark = pytest.mark.gpu

ROWSZ = 64 * 512 + 64  # words of one (o, lse) row in the exchange layout


def _wire(payload_f32: np.ndarray, epoch: int) -> np.ndarray:
    """The exchange's wire format: one 8-byte word {payload bits, epoch} per float."""
    bits = payload_f32.astype(np.float32).view(np.uint32).astype(np.uint64)
    return bits | (np.uint64(epoch) << np.uint64(32))


def _merge(region: torch.Tensor, slot_words: int, epoch_ctr: torch.Tensor, n_rows: int, n_parts: int):
    ctx = torch.full((n_rows, 64, 512), 7.0, dtype=torch.float32, device="cuda")
    lse = torch.full((n_rows, 64), 7.0, dtype=torch.float32, device="cuda")
    st = _lib.lib().wl_diag_merge_exchange(region.data_ptr(), slot_words, epoch_ctr.data_ptr(), n_rows, n_parts,
                                           ctx.data_ptr(), lse.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "wl_diag_merge_exchange")
    return ctx, lse


def test_exchange_consumer_merges_words_of_the_current_epoch():
    """The hook itself: parts in the wire format with the awaited epoch merge
    like the LSE merge of the split-K partials."""
    A.device_error(clear=True)
    rng = np.random.default_rng(3)
    n_rows, n_parts = 2, 3
    o_parts = rng.standard_normal((n_parts, n_rows, 64, 512)).astype(np.float32)
    l_parts = rng.uniform(-3, 3, (n_parts, n_rows, 64)).astype(np.float32)
    l_parts[1, 0, 5] = -np.inf  # an empty part of one head is skipped
    words = np.zeros((n_parts, n_rows, ROWSZ), np.uint64)
    for s in range(n_parts):
        for r in range(n_rows):
            words[s, r] = _wire(np.concatenate([o_parts[s, r].ravel(), l_parts[s, r]]), 5)
    region = torch.from_numpy(words.view(np.int64).reshape(-1)).cuda()
    epoch = torch.tensor([5], dtype=torch.int32, device="cuda")
    ctx, lse = _merge(region, n_rows * ROWSZ, epoch, n_rows, n_parts)
    torch.cuda.synchronize()
    assert A.device_error(clear=True)[0] == _lib.WL_OK
    m = l_parts.max(0)
    w = np.exp(l_parts - m[None])
    ref_l = m + np.log(w.sum(0))
    ref_o = (w[..., None] * o_parts).sum(0) / w.sum(0)[..., None]
    np.testing.assert_allclose(lse.cpu().numpy(), ref_l, rtol=0, atol=1e-5)
    np.testing.assert_allclose(ctx.cpu().numpy(), ref_o, rtol=1e-5, atol=1e-5)


def test_a_wait_that_runs_out_reports_timeout_and_the_gpu_stays_usable():
    A.device_error(clear=True)
    n_rows, n_parts = 1, 2
    # every word carries epoch 0, the consumer waits for epoch 1: it never arrives
    region = torch.zeros(n_parts * n_rows * ROWSZ, dtype=torch.int64, device="cuda")
    epoch = torch.tensor([1], dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().wl_diag_set_wait_limit(2_000_000))  # ~1 ms at the SM clock
    try:
        _merge(region, n_rows * ROWSZ, epoch, n_rows, n_parts)
        st, word = A.device_error(clear=True)
    finally:
        _lib.check(_lib.lib().wl_diag_set_wait_limit(0))  # back to the default (~1 s)
    assert st == _lib.WL_ERR_TIMEOUT, f"status {st}, word 0x{word:08x}"
    assert (word >> 24) == 6  # the timeout code, site in bits 16-23
    assert A.device_error(clear=False)[0] == _lib.WL_OK  # cleared
    # the same context still runs the substep correctly
    T, k = 1500, 256
    inp = o.make_inputs(T, 1, seq=4)
    d = lambda x, t: torch.from_numpy(np.ascontiguousarray(x)).cuda()[None].to(t)  # noqa: E731
    kv = A.LatentKV(d(inp["c_kv"], torch.bfloat16), d(inp["k_rot"], torch.bfloat16))
    keys = A.IndexKeys(d(inp["idx_bits"], torch.uint8), d(inp["idx_scale"], torch.float32))
    cfg = A.glm52_cfg(T, index_topk=k)
    out = A.attn_decode(cfg, kv, d(inp["q_abs"], torch.bfloat16), keys=keys, q_idx=d(inp["q_idx"], torch.bfloat16),
                        w_idx=d(inp["w_idx"], torch.float32))
    torch.cuda.synchronize()
    assert A.device_error(clear=True)[0] == _lib.WL_OK
    rc, _ = o.mla_sparse(inp["q_abs"], inp["c_kv"], inp["k_rot"], out["sel"].cpu().numpy()[0], 1 / 16)
    assert o.bf16_ulp_error(rc, out["ctx"].cpu().numpy()[0]) <= 2.0


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_sharded_exchange_layout_on_one_gpu(nranks):
    """The sharded decode's peer-memory combination of (o, lse) partials —
    reduce-scatter by heads, then all-gather — with `nranks` ranks emulated on
    one GPU (every stage runs for all ranks before the next one, so nothing
    waits on a kernel still to come): every rank must end with the merge of
    all ranks' split partials, equal to the merge kernel's on the same parts."""
    A.device_error(clear=True)
    L = _lib.lib()
    B, S = 3, 4
    rng = np.random.default_rng(nranks)
    o = rng.standard_normal((nranks, B, S, 64, 512)).astype(np.float32)
    lse = rng.uniform(-4, 4, (nranks, B, S, 64)).astype(np.float32)
    lse[0, 1, 2, 7] = -np.inf  # an empty split
    lse[:, 2, :, 9] = -np.inf  # a head with no keys anywhere
    lse[1 % nranks, 0, :, :] = -np.inf  # a rank whose window held none of row 0
    nb = L.wl_diag_xmerge_bytes(nranks)
    regions = torch.zeros(nb // 8 + 1, dtype=torch.int64, device="cuda")
    o_t, l_t = torch.from_numpy(o).cuda(), torch.from_numpy(lse).cuda()
    ctx = torch.full((nranks, B, 64, 512), 7.0, device="cuda")
    lo = torch.full((nranks, B, 64), 7.0, device="cuda")
    _lib.check(L.wl_diag_set_wait_limit(20_000_000))  # ~10 ms: a layout error times out quickly
    try:
        for call in range(2):  # the second call runs on the first call's slots (next epoch)
            _lib.check(L.wl_diag_xmerge(nranks, B, S, o_t.data_ptr(), l_t.data_ptr(), regions.data_ptr(), nb,
                                        ctx.data_ptr(), lo.data_ptr(), torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
            st, word = A.device_error(clear=True)
            assert st == _lib.WL_OK, f"call {call}: device error word 0x{word:08x}"
    finally:
        _lib.check(L.wl_diag_set_wait_limit(0))
    # reference: the merge kernel over all nranks * S parts of each row
    parts_o = torch.from_numpy(o.transpose(1, 0, 2, 3, 4).reshape(B, nranks * S, 64, 512)).cuda()
    parts_l = torch.from_numpy(lse.transpose(1, 0, 2, 3).reshape(B, nranks * S, 64)).cuda()
    ref_c, ref_l = A.lse_merge(parts_o, parts_l)
    for r in range(nranks):
        np.testing.assert_allclose(ctx[r].cpu().numpy(), ref_c.cpu().numpy(), rtol=1e-5, atol=1e-5)
        got_l, want_l = lo[r].cpu().numpy(), ref_l.cpu().numpy()
        assert np.array_equal(np.isinf(got_l), np.isinf(want_l))
        fin = np.isfinite(want_l)
        np.testing.assert_allclose(got_l[fin], want_l[fin], rtol=0, atol=1e-5)
