"""CPU oracle for the GLM-5.2 attention substep — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker / reported baseline. The
product path (``windlass_b200``) never calls it: it fails loudly when its CUDA
library is missing.

This is a numpy restatement of the reference's algorithm for the path, each
function citing the reference it follows (paths inside ssubbotin/windlass):

  indexer_scores   tools/ref_glm_chain.py:482-501   (relu between qk and the
                   head sum; two scales D^-0.5 and, folded into w, H^-0.5)
  indexer_topk     tools/ref_glm_chain.py:504-515   (min(k, T); stable argsort:
                   ties to the lowest index)
  index_drop_mask  tools/ref_glm_chain.py:518-529   (out-of-range indices
                   unmask nothing)
  mla_absorbed     src/glm_layer_runner.cuh:251-298 (absorbed form of
                   attn_block's s = q.K, drop -> -inf, softmax, p.V,
                   tools/ref_glm_chain.py:616-638)
  indexer_query    tools/ref_glm_chain.py:489-497 (indexer_scores' q and w:
                   wq_b @ q_resid, RoPE on the leading 64 of each head,
                   weights_proj @ x * H^-0.5; glm_kernels.cuh:469-472)
  mla_absorb_q     src/glm_layer_runner.cuh:196-215 (q_nope through W_UK),
                   with the roped part appended: the attention's input row
  mla_project_v    src/glm_layer_runner.cuh:217-234 (ctx through W_UV)
  lse_merge        the standard (o, lse) combination of disjoint key sets
  cache_append     the cache write path: indexer_keys (ref_glm_chain.py:
                   465-480; launch_indexer_key, src/glm_kernels.cuh:432-448)
                   and the latent row of attn_block (rms_norm + rope_interleave,
                   ref_glm_chain.py:63-106, 576-581; glm_layer_runner.cuh:
                   544-570), in the kernel's fixed summation order
  quantize_e4m3    the benchmark's fp8 index-key format (not in the reference):
                   e4m3 (OCP "fn", round-to-nearest-even) with one fp32 scale
                   per key = amax / 448.

The oracle is pinned against the reference itself: tests/golden/ holds
outputs of tools/ref_glm_indexer.py and of ref_glm_chain.attn_block run in
the build container (tests/golden/make_golden.py), and tests/test_oracle.py
checks these functions against them.
"""
from __future__ import annotations

import numpy as np

try:
    import ml_dtypes  # e4m3 rounding
    _E4M3 = ml_dtypes.float8_e4m3fn
except Exception:  # pragma: no cover - ml_dtypes ships with the image
    _E4M3 = None

E4M3_MAX = 448.0


# ---- bf16 / e4m3 helpers ----------------------------------------------------------------

def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit pattern, round-to-nearest-even (torch's cast)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rnd = ((u >> 16) & 1).astype(np.uint32) + np.uint32(0x7FFF)
    return ((u + rnd) >> 16).astype(np.uint16)


def from_bf16_bits(u: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return from_bf16_bits(to_bf16_bits(x))


def quantize_e4m3(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-row e4m3 quantisation: returns (uint8 bit patterns [T, D], scale [T] fp32)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=-1)
    scale = np.where(amax > 0, amax / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)
    q = (x / scale[..., None]).astype(np.float32)
    bits = q.astype(_E4M3).view(np.uint8)
    return bits, scale


def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint8).view(_E4M3).astype(np.float32)


def dequant_e4m3(bits: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Key values the indexer sees: e4m3(bits) * scale, in fp32."""
    return (e4m3_to_f32(bits) * np.asarray(scale, dtype=np.float32)[..., None]).astype(np.float32)


# ---- the hot path ------------------------------------------------------------------------

def indexer_scores(q: np.ndarray, K: np.ndarray, w: np.ndarray, D: int | None = None) -> np.ndarray:
    """index[t] = sum_h w[h] * relu((q[h] . K[t]) * D^-0.5)  (ref_glm_chain.py:482-501).

    q [H, D] fp32 (post-RoPE), K [T, D] fp32 (dequantised keys), w [H] fp32
    (already x H^-0.5, ref_glm_chain.py:499). Returns [T] fp32."""
    q = np.asarray(q, np.float32)
    K = np.asarray(K, np.float32)
    w = np.asarray(w, np.float32)
    D = q.shape[-1] if D is None else D
    s = np.maximum((q @ K.T) * np.float32(D ** -0.5), 0.0)
    return (w[:, None] * s).sum(0, dtype=np.float32)


def indexer_topk(index: np.ndarray, k: int) -> np.ndarray:
    """The selected keys (ref_glm_chain.py:504-515): argsort(-index, stable)[:min(k,T)]."""
    kk = min(k, index.shape[0])
    return np.argsort(-index, kind="stable")[:kk].astype(np.int32)


def index_drop_mask(sel: np.ndarray, T: int) -> np.ndarray:
    """True == DROP; indices outside [0, T) unmask nothing (ref_glm_chain.py:518-529)."""
    drop = np.ones(T, bool)
    sel = np.asarray(sel)
    drop[sel[(sel >= 0) & (sel < T)]] = False
    return drop


def canonical(sel: np.ndarray, T: int) -> np.ndarray:
    """The selection as the ascending list of kept keys."""
    return np.nonzero(~index_drop_mask(sel, T))[0].astype(np.int32)


def mla_absorbed(q_abs: np.ndarray, c_kv: np.ndarray, k_rot: np.ndarray, drop: np.ndarray | None,
                 scale: float, dtype=np.float64) -> tuple[np.ndarray, np.ndarray]:
    """Absorbed MLA attention of one query (glm_layer_runner.cuh:251-298).

    q_abs [H, L+R] (absorbed latent query | roped rope query), c_kv [T, L],
    k_rot [T, R], drop [T] bool (True = masked) or None. Returns
    ctx [H, L] and lse [H] (natural log of the softmax denominator of the
    scaled scores)."""
    L = c_kv.shape[1]
    q = np.asarray(q_abs, dtype)
    kv = np.asarray(c_kv, dtype)
    kr = np.asarray(k_rot, dtype)
    s = (q[:, :L] @ kv.T + q[:, L:] @ kr.T) * dtype(scale)  # [H, T]
    if drop is not None and drop.any():
        s = np.where(drop[None, :], -np.inf, s)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    z = p.sum(-1, keepdims=True)
    ctx = (p @ kv) / z
    lse = (m + np.log(z))[:, 0]
    return ctx, lse


def mla_sparse(q_abs, c_kv, k_rot, sel, scale, dtype=np.float64):
    """mla_absorbed over the keys `sel` keeps (gathering only those rows)."""
    T = c_kv.shape[0]
    keep = canonical(sel, T)
    return mla_absorbed(q_abs, c_kv[keep], k_rot[keep], None, scale, dtype)


def indexer_query(q_resid, wq_b, x, weights_proj, cos, sin, H: int = 32, D: int = 128, R: int = 64):
    """(q [n, H, D] post-RoPE, w [n, H]) for n query rows, float64: q = wq_b @ q_resid
    reshaped per head with RoPE (interleaved in, halves out) on its leading R
    dims; w = weights_proj @ x * H^-0.5 (ref_glm_chain.py:489-497)."""
    q = np.asarray(q_resid, np.float64) @ np.asarray(wq_b, np.float64).T
    q = q.reshape(q.shape[0], H, D)
    c, s = np.asarray(cos, np.float64)[:, None, :], np.asarray(sin, np.float64)[:, None, :]
    a, b = q[..., 0:R:2], q[..., 1:R:2]
    q = np.concatenate([a * c - b * s, b * c + a * s, q[..., R:]], axis=-1)
    w = np.asarray(x, np.float64) @ np.asarray(weights_proj, np.float64).T * H ** -0.5
    return q, w


def mla_absorb_q(q: np.ndarray, kv_b: np.ndarray, nope: int = 192, v_head: int = 256) -> np.ndarray:
    """q [..., H, nope + rope] (rope part already roped), kv_b [H * (nope + v_head), L]
    -> [..., H, L + rope]: sum_d q[h][d] kv_b[h*(nope+v_head) + d][c], then q[h][nope:]
    (glm_layer_runner.cuh:196-215; float64)."""
    q = np.asarray(q, np.float64)
    H = q.shape[-2]
    W = np.asarray(kv_b, np.float64).reshape(H, nope + v_head, -1)
    return np.concatenate([np.einsum("...hd,hdc->...hc", q[..., :nope], W[:, :nope]), q[..., nope:]], -1)


def mla_project_v(ctx: np.ndarray, kv_b: np.ndarray, nope: int = 192, v_head: int = 256) -> np.ndarray:
    """ctx [..., H, L] -> [..., H, v_head]: sum_c ctx[h][c] kv_b[h*(nope+v_head) + nope + v][c]
    (glm_layer_runner.cuh:217-234; float64)."""
    ctx = np.asarray(ctx, np.float64)
    H = ctx.shape[-2]
    W = np.asarray(kv_b, np.float64).reshape(H, nope + v_head, -1)
    return np.einsum("...hc,hvc->...hv", ctx, W[:, nope:])


def lse_merge(os: list[np.ndarray], lses: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    """Combine partial (ctx, lse) over disjoint key sets."""
    L = np.stack(lses)  # [S, H]
    M = L.max(0)
    Mf = np.where(np.isfinite(M), M, 0.0)
    wgt = np.where(np.isfinite(L), np.exp(L - Mf), 0.0)
    W = wgt.sum(0)
    o = sum(wgt[i][:, None] * os[i] for i in range(len(os))) / np.where(W > 0, W, 1.0)[:, None]
    return o, np.where(W > 0, Mf + np.log(np.where(W > 0, W, 1.0)), -np.inf)


# ---- the substep ---------------------------------------------------------------------------

def decode_step(inp: dict, k: int, mode: str = "owner", sel_in=None, dtype=np.float64):
    """One decode token of one sequence: owner -> scores, top-k, sparse attention;
    consumer -> attention over sel_in; dense -> over every key.

    inp: c_kv [T,512] f32, k_rot [T,64] f32, q_abs [64,576] f32, q_idx [32,128]
    f32, w_idx [32] f32, idx_bits [T,128] u8, idx_scale [T] f32, scale."""
    T = inp["c_kv"].shape[0]
    out = {}
    if mode == "owner":
        K = dequant_e4m3(inp["idx_bits"], inp["idx_scale"])
        idx = indexer_scores(inp["q_idx"], K, inp["w_idx"])
        sel = indexer_topk(idx, k)
        out.update(index=idx, sel=sel)
    elif mode == "consumer":
        if sel_in is None:
            raise RuntimeError("shared layer with no published indices")
        sel = np.asarray(sel_in)
    else:
        sel = np.arange(T, dtype=np.int32)
    ctx, lse = mla_sparse(inp["q_abs"], inp["c_kv"], inp["k_rot"], sel, inp["scale"], dtype)
    out.update(ctx=ctx, lse=lse)
    return out


def prefill_rows(inp: dict, pos0: int, n_q: int, k: int, rows=None, dtype=np.float64):
    """Per-row decode semantics of chunked prefill (run_prefill_layer_major,
    glm_layer_runner.cuh:963-983): row i sees keys [0, pos0+i] and selects its
    own top-k over exactly those. inp holds per-row q_abs [n_q,64,576],
    q_idx [n_q,32,128], w_idx [n_q,32] and the full caches."""
    K = dequant_e4m3(inp["idx_bits"], inp["idx_scale"])
    res = []
    for i in (range(n_q) if rows is None else rows):
        T = pos0 + i + 1
        idx = indexer_scores(inp["q_idx"][i], K[:T], inp["w_idx"][i])
        sel = indexer_topk(idx, k)
        ctx, lse = mla_sparse(inp["q_abs"][i], inp["c_kv"][:T], inp["k_rot"][:T], sel, inp["scale"], dtype)
        res.append(dict(index=idx, sel=sel, ctx=ctx, lse=lse))
    return res


def sharded_decode(inp: dict, k: int, nranks: int):
    """The sharded algorithm on one host: contiguous key shards, local top-k
    candidates, exact global selection from the candidates (ties to the lowest
    global index), per-shard partial attention, (o, lse) merge."""
    T = inp["c_kv"].shape[0]
    bounds = [(r * T // nranks, (r + 1) * T // nranks) for r in range(nranks)]
    K = dequant_e4m3(inp["idx_bits"], inp["idx_scale"])
    cs, ci = [], []
    for lo, hi in bounds:
        idx = indexer_scores(inp["q_idx"], K[lo:hi], inp["w_idx"])
        loc = np.sort(indexer_topk(idx, k))
        cs.append(idx[loc])
        ci.append(loc + lo)
    cs, ci = np.concatenate(cs), np.concatenate(ci)  # ascending global index
    glob = np.sort(ci[indexer_topk(cs, min(k, T))])
    os_, ls_ = [], []
    for lo, hi in bounds:
        mine = glob[(glob >= lo) & (glob < hi)] - lo
        if mine.size == 0:
            os_.append(np.zeros((inp["q_abs"].shape[0], inp["c_kv"].shape[1])))
            ls_.append(np.full(inp["q_abs"].shape[0], -np.inf))
            continue
        o, l = mla_absorbed(inp["q_abs"], inp["c_kv"][lo:hi][mine], inp["k_rot"][lo:hi][mine], None,
                            inp["scale"])
        os_.append(o)
        ls_.append(l)
    ctx, lse = lse_merge(os_, ls_)
    return dict(sel=glob, ctx=ctx, lse=lse)


# ---- the cache write path ------------------------------------------------------------------

def _lane_tree(p: np.ndarray) -> np.ndarray:
    """Sum of 32 per-lane fp32 partials [..., 32] in a warp's tree order:
    lanes l < o add lane l + o for o = 16, 8, 4, 2, 1; lane 0 holds the sum."""
    p = np.array(p, dtype=np.float32, copy=True)
    for o in (16, 8, 4, 2, 1):
        p[..., :o] = p[..., :o] + p[..., o:2 * o]
    return p[..., 0]


def _rope_halves(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    a, b = x[..., 0::2], x[..., 1::2]
    return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1).astype(np.float32)


def cache_append(k_raw, k_norm_w, k_norm_b, kv_raw, kv_norm_w, cos, sin, ln_eps=1e-6, rms_eps=1e-6) -> dict:
    """The cache rows of n tokens from the projections' outputs.

    Index key (indexer_keys, ref_glm_chain.py:465-480; glm_kernels.cuh:255-285):
    LayerNorm of k_raw [n, 128] (biased variance, eps ln_eps) with weight and
    bias, RoPE (interleaved in, halves out) on the leading 64 dims, rounded to
    bf16, then quantize_e4m3. Latent row (attn_block, ref_glm_chain.py:576-581
    and 596): rms_norm of kv_raw[:, :512] with the weight (eps rms_eps), RoPE
    of kv_raw[:, 512:], both rounded to bf16. cos/sin [n, 32] fp32.

    The formulas are the reference's; the order of the fp32 sums and of the
    roundings is the kernel's (lane l of a warp sums its elements in order,
    then the lanes combine as in _lane_tree; x - mean, then * inv, then * w,
    then + b), so the result matches the kernel to the bit. The reference's own
    order differs only within fp32 rounding (checked against its outputs in
    tests/test_oracle.py)."""
    f = np.float32
    cos, sin = np.asarray(cos, f), np.asarray(sin, f)
    out = {}
    k = np.asarray(k_raw, f)
    n = k.shape[0]
    ks = k.reshape(n, 32, 4)
    mean = _lane_tree(((ks[..., 0] + ks[..., 1]) + ks[..., 2]) + ks[..., 3]) / f(128)
    d = (k - mean[:, None]).astype(f)
    dd = (d * d).reshape(n, 32, 4)
    var = _lane_tree(((dd[..., 0] + dd[..., 1]) + dd[..., 2]) + dd[..., 3]) / f(128)
    inv = (f(1) / np.sqrt((var + f(ln_eps)).astype(f))).astype(f)
    y = ((d * inv[:, None]) * np.asarray(k_norm_w, f) + np.asarray(k_norm_b, f)).astype(f)
    key = np.concatenate([_rope_halves(y[:, :64], cos, sin), y[:, 64:]], axis=-1)
    out["key_f32"] = key
    out["key_bf16"] = bf16_round(key)
    out["idx_bits"], out["idx_scale"] = quantize_e4m3(out["key_bf16"])
    x = np.asarray(kv_raw, f)
    c = x[:, :512].reshape(n, 4, 32, 4)  # element j*128 + 4l + e
    acc = np.zeros((n, 32), f)
    for j in range(4):
        for e in range(4):
            acc = (acc + c[:, j, :, e] * c[:, j, :, e]).astype(f)
    ms = _lane_tree(acc) / f(512)
    inv = (f(1) / np.sqrt((ms + f(rms_eps)).astype(f))).astype(f)
    out["c_kv_f32"] = ((x[:, :512] * inv[:, None]) * np.asarray(kv_norm_w, f)).astype(f)
    out["c_kv"] = bf16_round(out["c_kv_f32"])
    out["k_rot_f32"] = _rope_halves(x[:, 512:576], cos, sin)
    out["k_rot"] = bf16_round(out["k_rot_f32"])
    return out


# ---- seeded inputs (benchmark configs) ------------------------------------------------------------

def rope_interleave(x: np.ndarray, pos: np.ndarray, theta: float) -> np.ndarray:
    """Interleaved-in, halves-out RoPE (ref_glm_chain.py:85-106), float64 tables."""
    rot = x.shape[-1]
    inv = 1.0 / (theta ** (np.arange(0, rot, 2, dtype=np.float64) / rot))
    ang = np.asarray(pos, np.float64)[:, None] * inv[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    a, b = x[..., 0::2], x[..., 1::2]
    return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1).astype(np.float32)


def make_inputs(T: int, config: int, seq: int = 0, n_q: int = 1, theta: float = 1e6) -> dict:
    """Seeded synthetic inputs with the benchmark's shapes and distributions.

    seed = 20260801 + config + 1000 * seq. c_kv ~ N(0,1) RMS-normalised per
    row; k_rot ~ N(0,1) roped at positions 0..T-1; q_abs, q_idx ~ N(0,1); all
    of those rounded to bf16. Index keys ~ N(0,1) quantised to e4m3 with a
    per-key scale; w ~ U(0,1). Arrays are float32 holding bf16-exact values;
    n_q > 1 gives per-row queries for prefill."""
    rng = np.random.default_rng(20260801 + config + 1000 * seq)
    ckv = rng.standard_normal((T, 512), dtype=np.float32)
    ckv = ckv / np.sqrt((ckv * ckv).mean(-1, keepdims=True) + 1e-6)
    krot = rope_interleave(rng.standard_normal((T, 64), dtype=np.float32), np.arange(T), theta)
    shape_q = (n_q,) if n_q > 1 else ()
    q_abs = rng.standard_normal(shape_q + (64, 576), dtype=np.float32)
    q_idx = rng.standard_normal(shape_q + (32, 128), dtype=np.float32)
    w = rng.uniform(0.0, 1.0, shape_q + (32,)).astype(np.float32)
    bits, scale = quantize_e4m3(rng.standard_normal((T, 128), dtype=np.float32))
    return dict(c_kv=bf16_round(ckv), k_rot=bf16_round(krot), q_abs=bf16_round(q_abs),
                q_idx=bf16_round(q_idx), w_idx=w, idx_bits=bits, idx_scale=scale,
                scale=1.0 / 16.0)


def bf16_ulp_error(ref: np.ndarray, got: np.ndarray) -> float:
    """Max |got - ref| in units of one bf16 ulp at the tensor's scale, 2^-8 max|ref|
    (the metric of the reference's layer test, src/test_glm_layer.cu:141-200)."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    unit = 2.0 ** -8 * np.abs(ref).max()
    return float(np.abs(got - ref).max() / unit) if unit > 0 else float(np.abs(got - ref).max())
