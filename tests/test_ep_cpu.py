"""Expert-parallel MoE data flow (lagunalab_b200/ep.py) on gloo CPU ranks.

Every rank runs CollectiveExpertParallel — the data flow of the peer-memory kernels: one send
per (token, owner) in token-order slots, local expert ids, per-pick bf16(y * w) returned to the
source's (token, pick) row, combine in pick order — with the oracle's arithmetic injected
(route = laguna.py:137-145, experts = SwitchGLU on the rank's slice, shared MLP = laguna.py:
114-122); the result must equal the single-process oracle block (laguna.py:147-150) on the
same tokens.
Covers world sizes 2 and 4, a rank with no tokens, routing that keeps every pick on the
source rank, the uneven-split error, and a rank that fails before the exchange (the others
must get an error from the process group, not hang).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_ref
from tests._util import COS_TOL, REL_TOL, cos, rel_err


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02
    return dict(gate=r(E, H), bias=torch.randn(E, generator=g) * 0.5,
                wg=r(E, I, H), wu=r(E, I, H), wd=r(E, H, I),
                sh=(r(I, H), r(I, H), r(H, I)))


def _tokens(T, H, rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(T, H, generator=g).to(torch.bfloat16)


def _worker(rank, W, port, cfg, results):
    from lagunalab_b200.ep import CollectiveExpertParallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=W,
                            timeout=datetime.timedelta(seconds=cfg.get("pg_timeout", 60)))
    try:
        E, k, H, I, scale = cfg["E"], cfg["k"], cfg["H"], cfg["I"], cfg["scale"]
        wts = _weights(E, H, I, seed=0)
        El = E // W if E % W == 0 else 1
        if cfg.get("local_only"):
            # a bias that sends every pick of rank r to rank r's own experts
            wts["bias"] = torch.full((E,), -1e4)
            wts["bias"][rank * El:(rank + 1) * El] = 0.0
        x = _tokens(cfg["T"][rank], H, rank)
        route_fn = lambda x2: moe_ref.route(x2, wts["gate"], wts["bias"], k)[:2]

        def expert_fn(rows, lid):
            inds = torch.where(lid >= 0, lid.to(torch.int64) + rank * El, -1)
            return moe_ref.switch_glu_deq(rows, inds, wts["wg"], wts["wu"], wts["wd"])

        shared_fn = lambda x2: moe_ref.mlp_deq(x2, *wts["sh"])
        if cfg.get("fail_rank") == rank:
            raise RuntimeError("planted failure before the exchange")
        ep = CollectiveExpertParallel(E, k, scale, route_fn, expert_fn, shared_fn,
                                      capacity=max(max(cfg["T"]), 1))
        out = ep(x)
        inds, w = route_fn(x)
        want = moe_ref.combine(moe_ref.switch_glu_deq(x, inds, wts["wg"], wts["wu"], wts["wd"]),
                               w, scale, shared_fn(x))
        results[rank] = ("ok", out.float(), want.float())
    except Exception as e:  # reported to the parent; a planted failure is expected
        results[rank] = ("error", repr(e), None)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(W, cfg, timeout=240):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        results = man.dict()
        port = _port()
        procs = [ctx.Process(target=_worker, args=(r, W, port, cfg, results)) for r in range(W)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        return {r: results[r] for r in results.keys()}


@pytest.mark.parametrize("W", [2, 4])
def test_ep_matches_single_process_block(W):
    cfg = dict(E=16, k=4, H=128, I=64, scale=2.5, T=[24, 17, 9, 31][:W])
    res = _run(W, cfg)
    assert sorted(res) == list(range(W))
    for r, (status, out, want) in res.items():
        assert status == "ok", out
        assert out.shape == want.shape
        assert rel_err(out, want) <= REL_TOL and cos(out, want) >= COS_TOL, r


def test_ep_rank_without_tokens_and_local_only_routing():
    res = _run(2, dict(E=8, k=2, H=64, I=64, scale=1.0, T=[12, 0]))
    for r, (status, out, want) in res.items():
        assert status == "ok", out
        assert out.shape[0] == [12, 0][r]
        if out.numel():
            assert rel_err(out, want) <= REL_TOL
    res = _run(2, dict(E=8, k=2, H=64, I=64, scale=1.0, T=[10, 7], local_only=True))
    for r, (status, out, want) in res.items():
        assert status == "ok", out
        assert rel_err(out, want) <= REL_TOL and cos(out, want) >= COS_TOL


def test_ep_uneven_expert_split_is_refused():
    res = _run(2, dict(E=9, k=2, H=64, I=64, scale=1.0, T=[4, 4]))
    for r, (status, msg, _) in res.items():
        assert status == "error" and "split evenly" in msg


def test_ep_failed_rank_ends_the_others_with_an_error():
    res = _run(2, dict(E=8, k=2, H=64, I=64, scale=1.0, T=[6, 6], fail_rank=1, pg_timeout=10),
               timeout=120)
    assert res[1][0] == "error" and "planted failure" in res[1][1]
    assert res[0][0] == "error"  # its exchange ended with an error instead of waiting forever


def test_balanced_placement_splits_evenly_and_balances():
    from lagunalab_b200 import ep
    counts = [1000, 900, 10, 10, 500, 400, 5, 5]
    pl = ep.balanced_placement(counts, 2)
    assert sorted(e for p in pl for e in p) == list(range(8)) and all(len(p) == 4 for p in pl)
    loads = [sum(counts[e] for e in p) for p in pl]
    assert max(loads) - min(loads) <= 200  # contiguous halves would be 1920 against 910
    with pytest.raises(ValueError):
        ep.balanced_placement(counts, 3)
