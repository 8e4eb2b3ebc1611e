"""GPU, two devices: failure detection of the peer-memory ZeRO-1 exchange,
made on the host (no GPU fault).  Both ranks take one reduced micro-step and
one AdamW step (which sets up the mappings and leaves both idle), then rank 1
stops taking part: it stays alive, with nothing in flight, until the test
ends.  Rank 0's next micro-step must not hold its GPU: the exchange kernels
that wait for rank 1's epoch flags give up at the wall-clock limit derived
from ne_comm_set_timeout, the call returns NE_ERR_TIMEOUT, and later exchanges
on that communicator are refused with NE_ERR_STATE.  NVLS is off in NCCL (used
here only to exchange the IPC handles); the exchange itself is plain peer
loads.  Skipped with fewer than two GPUs."""
import os
import time

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _cfg():
    from oracle import model as om
    return om.ModelCfg(n_layers=2, dim=128, hidden=256, heads=4, kv_heads=2, head_dim=64,
                       vocab=512, qk_norm=True, theta=1e6, eps=1e-6)


def _rank(rank, uid, tok, q, go):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["NE_COMM_PX"] = "1"
    import neural_engine_b200 as ne
    from oracle import model as om
    res = {"rank": rank}
    e = None
    try:
        torch.cuda.set_device(rank)
        cfg = _cfg()
        layers, rf, emb, qk = om.init_weights(cfg, seed=4, std=0.08, bf16=True)
        e = ne.Engine(cfg, device=rank)
        e.set_weights(layers, rf, emb, qk)
        e.train_alloc(2, tok.shape[1] - 1)
        e.comm_set_timeout(4000)
        e.comm_init(uid, rank, 2)
        e.comm_set_sharding(True)
        mine = tok[2 * rank:2 * rank + 2]
        e.train_fwd_bwd(mine)
        e.adamw_step(1, 1e-3, grad_scale=0.5)
        if rank == 0:
            t0 = time.time()
            try:
                e.train_fwd_bwd(mine)          # rank 1 never enters this exchange
                res["status"] = 0
            except ne.NeError as err:
                res["status"] = err.status
                res["msg"] = str(err)
            res["seconds"] = time.time() - t0
            try:
                e.train_fwd_bwd(mine)
                res["again"] = 0
            except ne.NeError as err:
                res["again"] = err.status
        else:
            res["status"] = "stopped"
    except Exception as ex:                    # report instead of hanging the parent
        res["error"] = repr(ex)
    q.put(res)
    go.wait(120)                               # keep the mapped memory alive until the end
    if e is not None:
        e.close()


def test_rank_that_stops_taking_part_times_out_the_exchange():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import neural_engine_b200 as ne
    from oracle import model as om
    tok = om.prompt_tokens(_cfg().vocab, 33, 8, batch=4)
    uid = ne.Engine.comm_unique_id()
    ctx = mp.get_context("spawn")
    q, go = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_rank, args=(r, uid, tok, q, go)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in range(2):
            r = q.get(timeout=240)
            res[r["rank"]] = r
    finally:
        go.set()
        for p in procs:
            p.join(timeout=60)
    assert "error" not in res[0] and "error" not in res[1], res
    assert res[1]["status"] == "stopped"
    assert res[0]["status"] == 6, res[0]            # NE_ERR_TIMEOUT
    assert res[0]["seconds"] <= 30, res[0]
    assert res[0]["again"] == 8, res[0]             # NE_ERR_STATE: the exchange was aborted
