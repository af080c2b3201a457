"""Generate the golden fixtures that pin the oracle to the reference itself.

Run in a container that has the reference checkout (it is not needed at test
time; the outputs are committed):

    python tests/golden/make_golden.py --ref <path to ssubbotin/windlass>

Writes two files next to this script:

  indexer_ref.npz  tools/ref_glm_indexer.py run unmodified (its defaults:
                   seed 20260801, T=1024, index_topk=512, scale 1.0):
                   ref_q [32*128] fp32, ref_k_bf16 [1024,128] uint16,
                   ref_w [32], ref_index [1024], ref_topk [512].
  cache_ref.npz    the cache write path at GLM-5.2's dimensions: the
                   reference's indexer_keys (wk -> LayerNorm -> RoPE on the
                   leading 64) and the latent row of attn_block (rms_norm of
                   the first 512 of kv_a_proj_with_mqa, RoPE of the trailing
                   64) for 16 tokens at scattered positions, with the
                   projections' outputs the kernel takes as inputs.
  query_ref.npz    the indexer's query side at GLM-5.2's dimensions: the
                   reference's indexer_scores (its q and w) for 4 rows whose
                   inputs (q_resid, x with hidden 1024, wq_b, weights_proj,
                   RoPE rows) are regenerated from seed 20260806 by
                   query_inputs() below; only the outputs are stored.
  chain_ref.npz    tools/ref_glm_chain.attn_block (the direct, non-absorbed
                   MLA form with the DSA indexer and IndexShare) run over
                   positions 0..T-1 of a two-layer group (layer 0 "full",
                   layer 1 "shared") at reduced head dimensions with seeded
                   random weights, plus the pre-attention intermediates the
                   absorbed form consumes, computed with the reference's own
                   primitives (rms_norm, rope_interleave).
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def indexer_fixture(ref: str) -> dict:
    with tempfile.TemporaryDirectory() as d:
        subprocess.run([sys.executable, os.path.join(ref, "tools", "ref_glm_indexer.py"), "--out", d],
                       check=True, stdout=subprocess.DEVNULL)
        load = lambda n: np.load(os.path.join(d, n + ".npy"))  # noqa: E731
        return dict(ref_q=load("ref_q"), ref_k_bf16=load("ref_k_bf16"), ref_w=load("ref_w"),
                    ref_index=load("ref_index"), ref_topk=load("ref_topk"))


def chain_fixture(ref: str) -> dict:
    sys.path.insert(0, os.path.join(ref, "tools"))
    import ref_glm_chain as R  # noqa: E402

    HN, NP, RP, VD, L = 4, 8, 4, 6, 16
    HID, QL, IH, ID, TOPK, T = 24, 12, 2, 8, 5, 12
    DH = NP + RP
    cfg = dict(n_heads=HN, qk_nope=NP, qk_rope=RP, v_head=VD, kv_lora=L, rms_eps=1e-5,
               indexer_types=["full", "shared"], index_heads=IH, index_dim=ID, index_topk=TOPK)
    rng = np.random.default_rng(20260801)
    f32 = lambda *s, sd=0.3: (rng.standard_normal(s) * sd).astype(np.float32)  # noqa: E731

    def layer_weights():
        return dict(input_layernorm=(1 + f32(HID, sd=0.1)), q_a_proj=f32(QL, HID),
                    q_a_layernorm=(1 + f32(QL, sd=0.1)), q_b_proj=f32(HN * DH, QL),
                    kv_a_proj_with_mqa=f32(L + RP, HID), kv_a_layernorm=(1 + f32(L, sd=0.1)),
                    kv_b_proj=f32(HN * (NP + VD), L), o_proj=f32(HID, HN * VD),
                    ix_wk=f32(ID, HID), ix_k_norm_w=(1 + f32(ID, sd=0.1)), ix_k_norm_b=f32(ID, sd=0.05),
                    ix_wq_b=f32(IH * ID, QL), ix_weights_proj=f32(IH, HID))

    Ws = [layer_weights(), layer_weights()]
    cos, sin = R.rope_tables(T, RP, 8e6)
    hs = f32(T, HID, sd=1.0)
    caches = [{"k": [], "v": []}, {"k": [], "v": []}]
    out = {"dims": np.array([HN, NP, RP, VD, L, HID, QL, IH, ID, TOPK, T])}
    taps = [[], []]
    for pos in range(T):
        share = R.IndexShare()
        for layer in (0, 1):
            tp = {}
            R.attn_block(hs[pos], Ws[layer], cfg, pos, cos, sin, caches[layer], layer, R._tapper(tp), share=share)
            taps[layer].append(tp)
    for layer in (0, 1):
        W = Ws[layer]
        pre = dict(q_nope=[], q_rot=[], kc=[], k_rot=[])
        for pos in range(T):
            x = R.rms_norm(hs[pos], W["input_layernorm"], cfg["rms_eps"])
            q_resid = R.rms_norm(x @ W["q_a_proj"].T, W["q_a_layernorm"], R.LORA_NORM_EPS)
            q = (q_resid @ W["q_b_proj"].T).reshape(HN, DH)
            ckv = x @ W["kv_a_proj_with_mqa"].T
            pre["q_nope"].append(q[:, :NP])
            pre["q_rot"].append(R.rope_interleave(q[:, NP:], cos[pos], sin[pos]))
            pre["kc"].append(R.rms_norm(ckv[:L], W["kv_a_layernorm"], R.LORA_NORM_EPS))
            pre["k_rot"].append(R.rope_interleave(ckv[L:], cos[pos], sin[pos]))
        for k, v in pre.items():
            out[f"l{layer}_{k}"] = np.stack(v).astype(np.float32)
        out[f"l{layer}_kv_b_proj"] = W["kv_b_proj"]
        out[f"l{layer}_o_proj"] = W["o_proj"]
        out[f"l{layer}_attn_out"] = np.stack([t["attn_out"] for t in taps[layer]]).astype(np.float32)
    # Indexer taps of the owner (layer 0); ragged per position -> padded.
    out["ix_q"] = np.stack([t["indexer_q"] for t in taps[0]]).astype(np.float32)
    out["ix_w"] = np.stack([t["indexer_w"] for t in taps[0]]).astype(np.float32)
    idx = np.full((T, T), np.nan, np.float32)
    sel = np.full((T, TOPK), -1, np.int32)
    for pos, t in enumerate(taps[0]):
        idx[pos, :pos + 1] = t["indexer_index_score"]
        sel[pos, :len(t["indexer_topk"])] = t["indexer_topk"]
    out["ix_index"] = idx
    out["ix_topk"] = sel
    out["ix_keys"] = np.stack(caches[0]["ik"]).astype(np.float32)
    return out


def cache_fixture(ref: str) -> dict:
    sys.path.insert(0, os.path.join(ref, "tools"))
    import ref_glm_chain as R  # noqa: E402

    from oracle.attn_ref import bf16_round  # noqa: E402

    n, HID = 16, 64
    rng = np.random.default_rng(20260805)
    f32 = lambda *s, sd=1.0: (rng.standard_normal(s) * sd).astype(np.float32)  # noqa: E731
    W = dict(ix_wk=f32(128, HID, sd=0.15), ix_k_norm_w=bf16_round(1 + f32(128, sd=0.1)),
             ix_k_norm_b=bf16_round(f32(128, sd=0.05)), kv_a_proj_with_mqa=f32(576, HID, sd=0.15),
             kv_a_layernorm=bf16_round(1 + f32(512, sd=0.1)))
    cfg = dict(qk_rope=64)
    pos = np.array([0, 1, 2, 3, 17, 100, 511, 1000, 2047, 4095, 8191, 12345, 40000, 65535, 100000, 131071])
    cos, sin = R.rope_tables(131072, 64, 1e6)
    x = f32(n, HID)
    ckv = x @ W["kv_a_proj_with_mqa"].T
    return dict(pos=pos.astype(np.int32), cos=cos[pos], sin=sin[pos],
                k_raw=(x.astype(np.float32) @ W["ix_wk"].T).astype(np.float32), kv_raw=ckv.astype(np.float32),
                k_norm_w=W["ix_k_norm_w"], k_norm_b=W["ix_k_norm_b"], kv_norm_w=W["kv_a_layernorm"],
                ref_key=R.indexer_keys(x, W, cfg, pos, cos, sin).astype(np.float32),
                ref_kc=R.rms_norm(ckv[:, :512], W["kv_a_layernorm"], R.LORA_NORM_EPS).astype(np.float32),
                ref_krot=R.rope_interleave(ckv[:, 512:], cos[pos], sin[pos]).astype(np.float32))


def query_inputs() -> dict:
    """Seeded inputs of query_ref.npz (also called by the tests)."""
    rng = np.random.default_rng(20260806)
    n, HID = 4, 1024
    f32 = lambda *s, sd=1.0: (rng.standard_normal(s) * sd).astype(np.float32)  # noqa: E731
    wq_b = f32(32 * 128, 2048, sd=0.02)
    wq_b = ((wq_b.view(np.uint32) + 0x7FFF + ((wq_b.view(np.uint32) >> 16) & 1)) & 0xFFFF0000).view(np.float32)
    ang = rng.uniform(0, 2 * np.pi, (n, 32))
    return dict(q_resid=f32(n, 2048), x=f32(n, HID), wq_b=wq_b, weights_proj=f32(32, HID, sd=0.05),
                cos=np.cos(ang).astype(np.float32), sin=np.sin(ang).astype(np.float32),
                pos=np.array([0, 5, 100, 4095]))


def query_fixture(ref: str) -> dict:
    sys.path.insert(0, os.path.join(ref, "tools"))
    import ref_glm_chain as R  # noqa: E402

    q = query_inputs()
    cfg = dict(index_heads=32, index_dim=128, qk_rope=64)
    W = dict(ix_wq_b=q["wq_b"], ix_weights_proj=q["weights_proj"])
    K = np.zeros((1, 128), np.float32)
    outs_q, outs_w = [], []
    for i in range(4):
        # indexer_scores takes cos/sin tables indexed by pos: a one-row table per call
        qq, ww, _ = R.indexer_scores(q["q_resid"][i], q["x"][i], K, W, cfg, 0, q["cos"][i:i + 1], q["sin"][i:i + 1])
        outs_q.append(qq)
        outs_w.append(ww)
    return dict(ref_q=np.stack(outs_q).astype(np.float32), ref_w=np.stack(outs_w).astype(np.float32))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("WINDLASS_REF", ""), help="reference checkout")
    ap.add_argument("--which", default="indexer,chain,cache,query", help="fixtures to write (comma-separated)")
    a = ap.parse_args()
    if not a.ref or not os.path.isdir(os.path.join(a.ref, "tools")):
        raise SystemExit("pass --ref <path to the reference checkout>")
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # the repository root, for oracle/
    which = set(a.which.split(","))
    if "indexer" in which:
        np.savez_compressed(os.path.join(HERE, "indexer_ref.npz"), **indexer_fixture(a.ref))
    if "chain" in which:
        np.savez_compressed(os.path.join(HERE, "chain_ref.npz"), **chain_fixture(a.ref))
    if "cache" in which:
        np.savez_compressed(os.path.join(HERE, "cache_ref.npz"), **cache_fixture(a.ref))
    if "query" in which:
        np.savez_compressed(os.path.join(HERE, "query_ref.npz"), **query_fixture(a.ref))
    print("wrote", HERE)


if __name__ == "__main__":
    main()
