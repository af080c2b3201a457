"""Run one small configuration of the substep a fixed number of times, for
profilers (ncu launch lists and per-kernel captures). No timing, no output
beyond a final line; the inputs are the bench's seeded synthetic ones.

    python -m windlass_b200.profile_case --case decode --batch 1 --T 32768 --iters 3
    python -m windlass_b200.profile_case --case prefill --pos0 1024 --n_q 1024 --iters 2
"""
from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=["decode", "consumer", "prefill"], default="decode")
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
    if a.case == "prefill":
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
