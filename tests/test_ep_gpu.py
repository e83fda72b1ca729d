"""Expert parallelism over NVLink peer memory (lagunalab_b200/ep.py PeerExpertParallel,
csrc/ep.cu) on 2 and 4 GPUs, one process per GPU.

Each rank routes its own tokens through the seed-0 Zipf-routed config-2 block with its expert
slice; the output must equal, bit for bit, the one-GPU block (``SparseMoeBlock.__call__``)
on the same tokens whenever both take the tensor-core product path (the exchange moves rows
and pick outputs without arithmetic, and the combine is the one-GPU combine); a rank with so
few tokens that the one-GPU block takes the GEMV path is held to the parity bar instead. Three forwards in a row (the epoch flags and buffer reuse),
one with fewer tokens than the capacity, and a rank with no tokens. Skipped when the box has
fewer GPUs than ranks.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, W, port, cfg, results):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=W,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    pe = None
    try:
        from lagunalab_b200 import _lib, ep, synth
        E, cap = cfg["E"], cfg["cap"]
        blk, _ = synth.moe_block(0, E, 8, cfg["H"], cfg["I"], cfg["I"], seed=0, zipf=True,
                                 routed_scaling_factor=cfg["scale"])
        placement = cfg.get("placement")
        pe = ep.PeerExpertParallel(blk, capacity=cap, timeout_s=10.0, placement=placement)
        rep = []
        for step, T in enumerate(cfg["T"][rank]):
            g = torch.Generator(device="cuda")
            g.manual_seed(1000 * step + rank)
            x = torch.randn(T, cfg["H"], generator=g, device="cuda").to(torch.bfloat16)
            got = pe(x)
            want = blk(x) if T else got
            torch.cuda.synchronize()
            # the owners take the tensor-core path (capacity above LG_MOE_GEMV_MAX_ROWS / (k + 1)
            # tokens); the one-GPU block takes it for its own T only above that too
            same_path = T == 0 or T * 9 > _lib.LG_MOE_GEMV_MAX_ROWS
            err = float((got.float() - want.float()).abs().max()) if T else 0.0
            rel = err / max(float(want.float().abs().max()), 1e-30) if T else 0.0
            rep.append((T, bool(torch.equal(got, want)), err, same_path, rel))
        results[rank] = ("ok", rep, pe.status())
    except Exception as e:
        results[rank] = ("error", repr(e), None)
    finally:
        if pe is not None:
            try:
                pe.close()
            except Exception:
                pass
        dist.destroy_process_group()


TOKENS = {2: [[1024, 700, 1024], [1024, 0, 333]],
          4: [[1024, 700, 1024], [1024, 0, 333], [17, 1024, 0], [512, 1, 1024]]}


@pytest.mark.parametrize("W,placed", [(2, False), (2, True), (4, False)])
def test_peer_expert_parallel_equals_one_gpu_block(W, placed):
    """``placed``: the experts spread over the ranks by a non-contiguous placement (interleaved,
    as ``ep.balanced_placement`` may give) instead of contiguous ranges."""
    if torch.cuda.device_count() < W:
        pytest.skip(f"needs {W} GPUs")
    cfg = dict(E=32, H=2048, I=1024, scale=2.5, cap=1024, T=TOKENS[W])
    if placed:
        cfg["placement"] = [[e for e in range(32) if (e * 7) % W == d] for d in range(W)]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        results = man.dict()
        port = _port()
        procs = [ctx.Process(target=_worker, args=(r, W, port, cfg, results)) for r in range(W)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        res = {r: results[r] for r in results.keys()}
    assert sorted(res) == list(range(W))
    for r, (status, rep, st) in res.items():
        assert status == "ok", rep
        assert st == 0, f"rank {r}: a bounded wait expired (status {st:#x})"
        for T, same, err, same_path, rel in rep:
            if same_path:  # the same products in the same order: bit for bit
                assert same, f"rank {r}, {T} tokens: differs from the one-GPU block by {err}"
            else:  # GEMV against tensor-core sums: the parity bar
                assert rel <= 2e-2, f"rank {r}, {T} tokens: max relative error {rel}"
