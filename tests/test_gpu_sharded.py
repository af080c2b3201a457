"""KV-sequence sharding over 2-8 GPUs through wl_attn_decode_sharded, with the
exchanges over NVLink peer memory and over NCCL (WL_NO_P2P=1).

Rank r holds keys [r*T/N, (r+1)*T/N) of every cache. The selection must equal
the single-GPU selection exactly (a key's score does not depend on where it
lives), and ctx must agree with the single-GPU result within 2 bf16 ulp of the
output scale — on every one of several consecutive owner and consumer steps
(the peer exchange tags each step with an epoch and alternates partial
buffers). Runs as child processes, one per GPU (2, 4 or 8); skipped with fewer GPUs."""
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


def _worker(rank, world, port, T, B, out_path, exchange):
    if exchange == "nccl":
        os.environ["WL_NO_P2P"] = "1"
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
    res = dict(p2p=np.array(int(comm.p2p)))
    for step in range(3):
        out = A.attn_decode_sharded(cfg, comm, lo, T, kv, q_abs, keys=keys, q_idx=q_idx, w_idx=w_idx)
        # consumer layers reusing the global selection (one, then two in a row)
        for c in range(1 + step % 2):
            con = A.attn_decode_sharded(cfg, comm, lo, T, kv, q_abs, mode=_lib.WL_MODE_CONSUMER, sel_in=out["sel"],
                                        sel_n_in=out["sel_n"], canonical=True)
            torch.cuda.synchronize()
            res[f"ctx_con{step}_{c}"] = con["ctx"].cpu().numpy()
        res[f"sel{step}"] = out["sel"].cpu().numpy()
        res[f"ctx{step}"] = out["ctx"].cpu().numpy()
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


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
@pytest.mark.parametrize("T", [20000, 100000])
def test_sharded_decode(tmp_path, T, exchange, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if world > 2 and T < 100000:
        pytest.skip("the larger worlds run the long context only")
    from oracle import attn_ref as o
    B = 2
    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(world, _free_port(), T, B, path, exchange), nprocs=world, start_method="spawn")
    rs = [dict(np.load(path + f".{r}.npz")) for r in range(world)]
    r0 = rs[0]
    for r in rs:
        assert int(r["err"]) == 0
        assert int(r["p2p"]) == (exchange == "p2p")
    for step in range(3):
        for s in range(B):
            sel = r0[f"sel{step}"][s]
            assert np.array_equal(sel, r0["sel1"][s]), f"step {step}: sharded selection differs from single-GPU"
            for r in rs:
                assert np.array_equal(sel, r[f"sel{step}"][s])
                assert o.bf16_ulp_error(r0["ctx1"][s], r[f"ctx{step}"][s]) <= 2.0
                for c in range(1 + step % 2):
                    assert o.bf16_ulp_error(r0["ctx1"][s], r[f"ctx_con{step}_{c}"][s]) <= 2.0
