"""KV-sequence sharding over 2 GPUs through wl_attn_decode_sharded (NCCL).

Rank r holds keys [r*T/2, (r+1)*T/2) of every cache. The selection must equal
the single-GPU selection exactly (a key's score does not depend on where it
lives), and ctx must agree with the single-GPU result within 2 bf16 ulp of the
output scale. Runs as two child processes; skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, B, out_path):
    import torch.distributed as dist

    from oracle import attn_ref as o
    from windlass_b200 import _lib
    from windlass_b200 import attn as A

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    inps = [o.make_inputs(T, 2, seq=s) for s in range(B)]
    lo, hi = rank * T // world, (rank + 1) * T // world
    d = lambda x, t: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(t)  # noqa: E731
    st = lambda k, a=None, b=None: np.stack([i[k][a:b] if a is not None else i[k] for i in inps])  # noqa: E731
    kv = A.LatentKV(d(st("c_kv", lo, hi), torch.bfloat16), d(st("k_rot", lo, hi), torch.bfloat16))
    keys = A.IndexKeys(d(st("idx_bits", lo, hi), torch.uint8), d(st("idx_scale", lo, hi), torch.float32))
    q_abs, q_idx, w_idx = d(st("q_abs"), torch.bfloat16), d(st("q_idx"), torch.bfloat16), d(st("w_idx"), torch.float32)
    cfg = A.glm52_cfg(T)
    comm = A.Comm(rank, world)
    out = A.attn_decode_sharded(cfg, comm, lo, T, kv, q_abs, keys=keys, q_idx=q_idx, w_idx=w_idx)
    torch.cuda.synchronize()
    res = dict(sel=out["sel"].cpu().numpy(), ctx=out["ctx"].cpu().numpy(), lse=out["lse"].cpu().numpy())
    # consumer layer reusing the global selection
    con = A.attn_decode_sharded(cfg, comm, lo, T, kv, q_abs, mode=_lib.WL_MODE_CONSUMER, sel_in=out["sel"],
                                sel_n_in=out["sel_n"], canonical=True)
    torch.cuda.synchronize()
    res["ctx_con"] = con["ctx"].cpu().numpy()
    st_, word = A.device_error(clear=True)
    res["err"] = st_
    if rank == 0:
        # single-GPU reference through wl_attn_decode on the full caches
        kvf = A.LatentKV(d(st("c_kv"), torch.bfloat16), d(st("k_rot"), torch.bfloat16))
        kf = A.IndexKeys(d(st("idx_bits"), torch.uint8), d(st("idx_scale"), torch.float32))
        one = A.attn_decode(cfg, kvf, q_abs, keys=kf, q_idx=q_idx, w_idx=w_idx)
        res["sel1"] = one["sel"].cpu().numpy()
        res["ctx1"] = one["ctx"].cpu().numpy()
    np.savez(out_path + f".{rank}.npz", **res)
    comm.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("T", [20000, 100000])
def test_sharded_decode_two_gpus(tmp_path, T):
    from oracle import attn_ref as o
    B = 2
    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(2, _free_port(), T, B, path), nprocs=2, start_method="spawn")
    r0, r1 = (dict(np.load(path + f".{r}.npz")) for r in range(2))
    assert int(r0["err"]) == 0 and int(r1["err"]) == 0
    for s in range(B):
        assert np.array_equal(r0["sel"][s], r0["sel1"][s]), "sharded selection differs from single-GPU"
        assert np.array_equal(r0["sel"][s], r1["sel"][s])
        assert o.bf16_ulp_error(r0["ctx1"][s], r0["ctx"][s]) <= 2.0
        assert o.bf16_ulp_error(r0["ctx1"][s], r1["ctx"][s]) <= 2.0
        assert o.bf16_ulp_error(r0["ctx"][s], r0["ctx_con"][s]) <= 2.0
