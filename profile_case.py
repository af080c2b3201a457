"""Run one small configuration of the substep a fixed number of times, for
profilers (ncu launch lists and per-kernel captures). No timing, no output
beyond a final line; the inputs are the bench's seeded synthetic ones.

    python profile_case.py --case decode --batch 1 --T 32768 --iters 3
    python profile_case.py --case prefill --pos0 1024 --n_q 1024 --iters 2
    python profile_case.py --case around --batch 8 --iters 3
"""
from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=["decode", "consumer", "prefill", "around"], default="decode")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--T", type=int, default=32768)
    ap.add_argument("--pos0", type=int, default=1024)
    ap.add_argument("--n_q", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()

    import torch

    from bench import make_device_inputs
    from windlass_b200 import _lib
    from windlass_b200 import attn as A

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.case == "around":
        # the entry points either side of the substep, at a decode batch
        cfg = A.glm52_cfg(8192)
        g = torch.Generator(device=dev)
        g.manual_seed(11)
        B = a.batch
        kvb = (torch.randn(64 * 448, 512, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        wq = (torch.randn(4096, 2048, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        wp = torch.randn(32, 6144, device=dev, generator=g) * 0.02
        q, ctx = torch.randn(B, 64, 256, device=dev, generator=g), torch.randn(B, 64, 512, device=dev, generator=g)
        qr, xh = torch.randn(B, 2048, device=dev, generator=g), torch.randn(B, 6144, device=dev, generator=g)
        cs, sn = torch.rand(B, 32, device=dev, generator=g), torch.rand(B, 32, device=dev, generator=g)
        keys = A.IndexKeys(torch.zeros(B, 8192, 128, dtype=torch.uint8, device=dev),
                           torch.zeros(B, 8192, dtype=torch.float32, device=dev))
        kv = A.LatentKV.packed(torch.zeros(B, 8192, 576, dtype=torch.bfloat16, device=dev))
        pos = torch.full((B,), 8191, dtype=torch.int32, device=dev)
        seq = torch.arange(B, dtype=torch.int32, device=dev)
        ones = torch.ones(512, dtype=torch.bfloat16, device=dev)
        for _ in range(a.iters):
            A.indexer_query(cfg, qr, wq, xh, wp, cs, sn)
            A.cache_append(cfg, pos, cs, sn, keys=keys, k_raw=torch.randn(B, 128, device=dev, generator=g),
                           k_norm_w=ones[:128], k_norm_b=torch.zeros_like(ones[:128]), kv=kv,
                           kv_raw=torch.randn(B, 576, device=dev, generator=g), kv_norm_w=ones, seq=seq)
            A.mla_absorb_q(cfg, q, kvb)
            A.mla_project_v(cfg, ctx, kvb)
    elif a.case == "prefill":
        T = a.pos0 + a.n_q
        cfg = A.glm52_cfg(T)
        d = make_device_inputs(torch, 1, T, 0, 20260803, dev, n_q=a.n_q)
        for _ in range(a.iters):
            A.attn_prefill(cfg, d["kv"], d["q_abs"], a.pos0, keys=d["keys"], q_idx=d["q_idx"], w_idx=d["w_idx"])
    else:
        cfg = A.glm52_cfg(a.T)
        d = make_device_inputs(torch, a.batch, a.T, 0, 20260805, dev)
        own = A.attn_decode(cfg, d["kv"], d["q_abs"], keys=d["keys"], q_idx=d["q_idx"], w_idx=d["w_idx"])
        for _ in range(a.iters):
            if a.case == "decode":
                A.attn_decode(cfg, d["kv"], d["q_abs"], keys=d["keys"], q_idx=d["q_idx"], w_idx=d["w_idx"])
            else:
                A.attn_decode(cfg, d["kv"], d["q_abs"], mode=_lib.WL_MODE_CONSUMER, sel_in=own["sel"],
                              sel_n_in=own["sel_n"], canonical=True)
    torch.cuda.synchronize()
    st, word = A.device_error(clear=True)
    _lib.check(st, f"device error word 0x{word:08x}")
    print(f"profile_case {a.case} done")


if __name__ == "__main__":
    main()
