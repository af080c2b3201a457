"""The oracle, pinned against outputs of the reference itself (tests/golden/),
plus the properties the GPU tests rely on. CPU only."""
import os

import numpy as np
import pytest

from oracle import attn_ref as o

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(ref, got):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / (np.abs(ref).max() + 1e-300))


# ---- pin 1: tools/ref_glm_indexer.py fixtures (seed 20260801, T=1024, k=512) ----

@pytest.fixture(scope="module")
def ix():
    return dict(np.load(os.path.join(GOLD, "indexer_ref.npz")))


def test_indexer_scores_match_reference_fixture(ix):
    q = ix["ref_q"].reshape(32, 128)
    K = o.from_bf16_bits(ix["ref_k_bf16"]).reshape(-1, 128)
    got = o.indexer_scores(q, K, ix["ref_w"])
    # The reference kernel's fp32 arithmetic gate is 1e-5 (test_glm_indexer.cu:167).
    assert rel(ix["ref_index"], got) < 1e-6


def test_indexer_topk_matches_reference_fixture(ix):
    q = ix["ref_q"].reshape(32, 128)
    K = o.from_bf16_bits(ix["ref_k_bf16"]).reshape(-1, 128)
    sel = o.indexer_topk(o.indexer_scores(q, K, ix["ref_w"]), 512)
    assert set(sel.tolist()) == set(ix["ref_topk"].tolist())
    # and on the reference's own scores, index for index (same stable argsort)
    assert np.array_equal(o.indexer_topk(ix["ref_index"], 512), ix["ref_topk"])


def test_topk_k_at_least_T_is_every_key(ix):
    sel = o.indexer_topk(ix["ref_index"], 4096)
    assert sorted(sel.tolist()) == list(range(1024))


def test_negative_control_relu_after_combination_is_detected(ix):
    """relu applied after the head sum is a different function (ref_glm_indexer.py
    defect 'relu_after'): the gate must separate it from the reference."""
    q = ix["ref_q"].reshape(32, 128)
    K = o.from_bf16_bits(ix["ref_k_bf16"]).reshape(-1, 128)
    wrong = np.maximum((ix["ref_w"][:, None] * ((q @ K.T) * 128 ** -0.5)).sum(0), 0)
    assert rel(ix["ref_index"], wrong) > 1e-3


# ---- pin 2: ref_glm_chain.attn_block (direct form) vs the absorbed restatement ----

@pytest.fixture(scope="module")
def ch():
    return dict(np.load(os.path.join(GOLD, "chain_ref.npz")))


def _absorbed_attn_out(ch, layer, pos, sel, drop_mask=True):
    HN, NP, RP, VD, L, HID, QL, IH, ID, TOPK, T = ch["dims"].tolist()
    kvb = ch[f"l{layer}_kv_b_proj"]
    q = np.concatenate([ch[f"l{layer}_q_nope"][pos], ch[f"l{layer}_q_rot"][pos]], -1)
    q_abs = o.mla_absorb_q(q, kvb, nope=NP, v_head=VD)
    n = pos + 1
    drop = o.index_drop_mask(sel, n) if drop_mask else None
    ctx, _ = o.mla_absorbed(q_abs, ch[f"l{layer}_kc"][:n], ch[f"l{layer}_k_rot"][:n], drop, (NP + RP) ** -0.5)
    v = o.mla_project_v(ctx, kvb, nope=NP, v_head=VD).reshape(HN * VD)
    return v @ ch[f"l{layer}_o_proj"].T


@pytest.mark.parametrize("layer", [0, 1])
def test_absorbed_attention_matches_reference_attn_block(ch, layer):
    T = int(ch["dims"][-1])
    for pos in range(T):
        sel = ch["ix_topk"][pos]
        sel = sel[sel >= 0]
        got = _absorbed_attn_out(ch, layer, pos, sel)
        assert rel(ch[f"l{layer}_attn_out"][pos], got) < 2e-5, (layer, pos)


def test_negative_control_mask_reaches_the_arithmetic(ch):
    """Above index_topk, ignoring the selection must change attn_out."""
    TOPK, T = int(ch["dims"][9]), int(ch["dims"][10])
    pos = T - 1
    assert pos + 1 > TOPK
    sel = ch["ix_topk"][pos]
    dense = _absorbed_attn_out(ch, 0, pos, sel[sel >= 0], drop_mask=False)
    assert rel(ch["l0_attn_out"][pos], dense) > 1e-3


def test_indexer_restatement_matches_attn_block_taps(ch):
    T = int(ch["dims"][-1])
    TOPK = int(ch["dims"][9])
    for pos in range(T):
        got = o.indexer_scores(ch["ix_q"][pos], ch["ix_keys"][:pos + 1], ch["ix_w"][pos])
        assert rel(ch["ix_index"][pos, :pos + 1], got) < 1e-6
        sel = o.indexer_topk(got, TOPK)
        ref = ch["ix_topk"][pos]
        assert set(sel.tolist()) == set(ref[ref >= 0].tolist())


def test_shared_layer_consumes_owner_selection(ch):
    """Layer 1 ("shared") attended over layer 0's selection: its attn_out is
    reproduced with layer 0's indices and not with dense attention."""
    TOPK, T = int(ch["dims"][9]), int(ch["dims"][10])
    pos = T - 1
    sel = ch["ix_topk"][pos]
    sel = sel[sel >= 0]
    assert rel(ch["l1_attn_out"][pos], _absorbed_attn_out(ch, 1, pos, sel)) < 2e-5
    assert rel(ch["l1_attn_out"][pos], _absorbed_attn_out(ch, 1, pos, sel, drop_mask=False)) > 1e-3


# ---- pin 3: the cache write path (indexer_keys and attn_block's latent row) ----

def test_cache_append_matches_reference_fixture():
    """The restatement (fixed fp32 summation order) against the reference's
    numpy at GLM-5.2's dimensions: fp32 rows within fp32 rounding, the RoPE
    part exact, and every stored bf16 / e4m3 value and scale identical to the
    same format applied to the reference's rows."""
    g = dict(np.load(os.path.join(GOLD, "cache_ref.npz")))
    r = o.cache_append(g["k_raw"], g["k_norm_w"], g["k_norm_b"], g["kv_raw"], g["kv_norm_w"], g["cos"], g["sin"])
    assert rel(g["ref_key"], r["key_f32"]) <= 1e-6
    assert rel(g["ref_kc"], r["c_kv_f32"]) <= 1e-6
    assert np.array_equal(g["ref_krot"], r["k_rot_f32"])
    bits, scale = o.quantize_e4m3(o.bf16_round(g["ref_key"]))
    assert np.array_equal(bits, r["idx_bits"]) and np.array_equal(scale, r["idx_scale"])
    assert np.array_equal(o.bf16_round(g["ref_kc"]), r["c_kv"])
    assert np.array_equal(o.bf16_round(g["ref_krot"]), r["k_rot"])


def test_cache_append_negative_control_layernorm_bias():
    """Dropping the LayerNorm bias (reusing an RMSNorm-like form for the
    indexer key) is visible at the fixture's tolerance."""
    g = dict(np.load(os.path.join(GOLD, "cache_ref.npz")))
    r = o.cache_append(g["k_raw"], g["k_norm_w"], np.zeros_like(g["k_norm_b"]), g["kv_raw"], g["kv_norm_w"],
                       g["cos"], g["sin"])
    assert rel(g["ref_key"], r["key_f32"]) > 1e-3


def test_cache_append_zero_key_gets_unit_scale():
    """A key whose LayerNorm output is all zero (zero weight, zero bias) is
    stored as e4m3 zeros with scale 1 (the format's amax = 0 rule)."""
    rng = np.random.default_rng(3)
    r = o.cache_append(rng.standard_normal((2, 128)).astype(np.float32), np.zeros(128, np.float32),
                       np.zeros(128, np.float32), rng.standard_normal((2, 576)).astype(np.float32),
                       np.ones(512, np.float32), np.ones((2, 32), np.float32), np.zeros((2, 32), np.float32))
    assert np.all(r["idx_bits"] == 0) and np.all(r["idx_scale"] == 1.0)
    # RoPE at angle 0 (cos 1, sin 0) only moves the pairs into the halves layout
    x = rng.standard_normal((2, 576)).astype(np.float32)
    r = o.cache_append(np.zeros((2, 128), np.float32), np.ones(128, np.float32), np.zeros(128, np.float32), x,
                       np.ones(512, np.float32), np.ones((2, 32), np.float32), np.zeros((2, 32), np.float32))
    assert np.array_equal(r["k_rot_f32"], np.concatenate([x[:, 512::2], x[:, 513::2]], -1))


# ---- pin 4: the indexer's query side (indexer_scores' q and w) ----

def test_indexer_query_matches_reference_fixture():
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import query_inputs

    q = query_inputs()
    g = dict(np.load(os.path.join(GOLD, "query_ref.npz")))
    rq, rw = o.indexer_query(q["q_resid"], q["wq_b"], q["x"], q["weights_proj"], q["cos"], q["sin"])
    assert rel(g["ref_q"], rq) <= 1e-6
    assert rel(g["ref_w"], rw) <= 1e-6
    # negative control: RoPE on the trailing 64 dims instead of the leading 64
    wrong = np.concatenate([rq[..., 64:], rq[..., :64]], -1)
    assert rel(g["ref_q"], wrong) > 1e-2


# ---- properties ----------------------------------------------------------------------

def test_e4m3_quantisation_roundtrip():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, 128)).astype(np.float32)
    bits, scale = o.quantize_e4m3(x)
    back = o.dequant_e4m3(bits, scale)
    assert bits.dtype == np.uint8 and scale.shape == (64,)
    assert np.abs(back).max(-1).tolist() == pytest.approx(np.abs(x).max(-1).tolist(), rel=1e-6)
    assert np.all(np.abs(back - x) <= np.abs(x) * 2 ** -4 + scale[:, None] * 2 ** -9 + 1e-12)


def test_drop_mask_out_of_range_unmasks_nothing():
    d = o.index_drop_mask(np.array([0, 1, 2, 10, -1]), 4)
    assert d.tolist() == [False, False, False, True]


def test_lse_merge_equals_whole():
    inp = o.make_inputs(300, 0)
    whole, lw = o.mla_absorbed(inp["q_abs"], inp["c_kv"], inp["k_rot"], None, 1 / 16)
    parts = [(0, 100), (100, 101), (101, 300)]
    os_, ls_ = zip(*[o.mla_absorbed(inp["q_abs"], inp["c_kv"][a:b], inp["k_rot"][a:b], None, 1 / 16)
                     for a, b in parts])
    m, lm = o.lse_merge(list(os_), list(ls_))
    assert np.abs(m - whole).max() < 1e-12 and np.abs(lm - lw).max() < 1e-12


@pytest.mark.parametrize("nranks", [2, 3, 4])
def test_sharded_algorithm_equals_single_gpu(nranks):
    inp = o.make_inputs(1500, 2)
    single = o.decode_step(inp, 256)
    sh = o.sharded_decode(inp, 256, nranks)
    assert np.array_equal(np.sort(single["sel"]), sh["sel"])
    assert np.abs(single["ctx"] - sh["ctx"]).max() < 1e-12


def test_sharded_ties_resolve_to_lowest_global_index():
    inp = o.make_inputs(64, 0)
    inp["w_idx"] = np.zeros_like(inp["w_idx"])  # every score is exactly 0: all ties
    sh = o.sharded_decode(inp, 10, 4)
    assert sh["sel"].tolist() == list(range(10))


def test_prefill_rows_are_causal():
    inp = o.make_inputs(40, 3, n_q=8)
    rows = o.prefill_rows(inp, 32, 8, 16)
    for i, r in enumerate(rows):
        assert r["sel"].max() <= 32 + i and len(r["sel"]) == 16
        assert r["index"].shape == (33 + i,)


def test_dense_equals_sparse_below_topk():
    inp = o.make_inputs(100, 0)
    a = o.decode_step(inp, 2048, "owner")
    b = o.decode_step(inp, 2048, "dense")
    assert np.array_equal(a["ctx"], b["ctx"])
