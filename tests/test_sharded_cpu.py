"""Host-side logic of the sharded path on CPU: two gloo ranks each score and
select on their own key shard, exchange (score, global index) candidates with
all_gather, select the exact global top-k (ties to the lowest global index),
attend over their part and merge the (o, lse) partials with a second
all_gather — and must reproduce the single-process result. Also: a rank that
dies before the exchange makes the other rank's collective fail (timeout)
instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, T, k, out):
    import torch.distributed as dist

    from oracle import attn_ref as o
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    inp = o.make_inputs(T, 2)
    lo, hi = rank * T // world, (rank + 1) * T // world
    K = o.dequant_e4m3(inp["idx_bits"][lo:hi], inp["idx_scale"][lo:hi])
    idx = o.indexer_scores(inp["q_idx"], K, inp["w_idx"])
    kl = min(k, hi - lo)
    loc = np.sort(o.indexer_topk(idx, k))
    cs = np.full(k, -np.inf, np.float32)
    ci = np.full(k, np.iinfo(np.int32).max, np.int64)
    cs[:kl], ci[:kl] = idx[loc], loc + lo
    gs = [torch.empty(k) for _ in range(world)]
    gi = [torch.empty(k, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gs, torch.from_numpy(cs))
    dist.all_gather(gi, torch.from_numpy(ci))
    cand_s = torch.cat(gs).numpy()
    cand_i = torch.cat(gi).numpy()
    glob = np.sort(cand_i[o.indexer_topk(cand_s, min(k, T))])
    mine = glob[(glob >= lo) & (glob < hi)] - lo
    if mine.size:
        oo, ll = o.mla_absorbed(inp["q_abs"], inp["c_kv"][lo:hi][mine], inp["k_rot"][lo:hi][mine], None, 1 / 16)
    else:
        oo, ll = np.zeros((64, 512)), np.full(64, -np.inf)
    po = [torch.empty(64, 512, dtype=torch.float64) for _ in range(world)]
    pl = [torch.empty(64, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(po, torch.from_numpy(np.ascontiguousarray(oo)))
    dist.all_gather(pl, torch.from_numpy(np.ascontiguousarray(ll)))
    ctx, lse = o.lse_merge([p.numpy() for p in po], [p.numpy() for p in pl])
    np.savez(out + f".{rank}.npz", sel=glob, ctx=ctx, lse=lse)
    dist.destroy_process_group()


@pytest.mark.parametrize("T,k", [(3000, 256), (900, 2048), (5000, 1)])
def test_two_rank_sharding_equals_single_process(tmp_path, T, k):
    from oracle import attn_ref as o
    path = str(tmp_path / "r")
    mp.start_processes(_rank, args=(2, _port(), T, k, path), nprocs=2, start_method="spawn")
    single = o.decode_step(o.make_inputs(T, 2), k)
    for r in range(2):
        res = np.load(path + f".{r}.npz")
        assert np.array_equal(res["sel"], np.sort(single["sel"]))
        assert np.abs(res["ctx"] - single["ctx"]).max() < 1e-10


def _dying(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the candidate exchange
    t = [torch.empty(4) for _ in range(world)]
    try:
        dist.all_gather(t, torch.ones(4))
        open(out, "w").write("completed")
    except Exception as e:  # the surviving rank learns of it from the collective
        open(out, "w").write("failed: " + type(e).__name__)


def test_rank_loss_fails_the_exchange_instead_of_hanging(tmp_path):
    out = str(tmp_path / "o.txt")
    ctx = mp.start_processes(_dying, args=(2, _port(), out), nprocs=2, start_method="spawn", join=False)
    ctx.processes[0].join(60)
    assert not ctx.processes[0].is_alive()
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert open(out).read().startswith("failed")
