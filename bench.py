"""Benchmark of the Laguna decoder hot path on B200 (the MoE block, the fused 8-bit KV decode
attention, and the bs1 decoder they sit in).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode_q8|decode|moe_prefill|moe_decode|q8_decode]

Prints ONE JSON line on rank 0. Default workload ``decode_q8`` (the headline metric): the
config-3 decoder (40 layers, 64 experts top-8, 4-bit g64 weights) decoding one token per step
at an 82,671-token context over the 8-bit quantized KV cache, each step one CUDA-graph replay;
metric tokens/s. ``decode`` is config 3 as stated (8,192-token prefill, bf16 KV);
``moe_prefill`` is config 2 (one MoE block on 4,096 Zipf-routed tokens, 128 experts, metric
"MoE-layer tokens/s"); ``moe_decode`` is config 1 (T = 16, graph-replayed); ``q8_decode`` is
config 4 (40 layers of fused 8-bit KV decode attention at 82,671 keys, HBM GB/s).

Timing: W warm-up steps, then K steps bracketed by a barrier and cuda synchronize, timed with
CUDA events on the launching stream; the max over ranks is reported. Inputs are resident in
HBM and larger than L2. ``e2e`` is the same metric through the public module API with the
step's input copied from pinned host memory and the output copied back inside the timed
region.

Multi-GPU (torchrun, N > 1): decode workloads run N independent replicas; the MoE workloads
run expert parallel (E/N experts per rank, NVLink peer-memory dispatch and return). Every line
also carries ``ep_prefill``: BASELINE config 5's 32,768-token MoE-layer prefill split over the
N ranks, with the one-GPU block as baseline and checker. ``--impl reference`` times the CPU
restatement of the reference's path on the host cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    "moe_prefill": dict(T=4096, E=128, k=8, H=2048, I=1024, I_sh=1024, zipf=True, scale=1.0),
    "moe_decode": dict(T=16, E=128, k=8, H=2048, I=1024, I_sh=1024, zipf=False, scale=2.5),
    "q8_decode": dict(L=40, n=82671, B=1, Hq=32, Hkv=4),
    # the 50%-pruned decoder, bs1 greedy decode after an 8,192-token prefill
    "decode": dict(prefill=8192, new=256, seed=1, vocab=100352, hidden=2048, layers=40, heads=32,
                   kv_heads=4, head_dim=128, experts=64, top_k=8, moe_inter=1024,
                   shared_inter=1024, dense_inter=8192, rope_theta=1e6, kv="bf16"),
    # the headline: the same decoder, bs1 greedy decode at an 82,671-token context over the
    # 8-bit quantized KV cache (DequantKVCache with fused_decode; BASELINE config 4's context)
    "decode_q8": dict(prefill=82671, new=256, seed=1, vocab=100352, hidden=2048, layers=40,
                      heads=32, kv_heads=4, head_dim=128, experts=64, top_k=8, moe_inter=1024,
                      shared_inter=1024, dense_inter=8192, rope_theta=1e6, kv="q8"),
}
DECODE_WORKLOADS = ("decode", "decode_q8")


def profile_traffic(name):
    """DRAM bytes per launch from the committed ncu summary profiles/<name>.md (the
    ``traffic_bytes_per_launch:`` line), or None."""
    p = ROOT / "profiles" / f"{name}.md"
    if p.exists():
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1])
    return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


# ----------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------

def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.idx = gpu_index
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        self.t0 = self.t1 = None

    def mark(self, start):
        if start:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def result(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        load = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ----------------------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------------------

def timed(step, K, stream, profile_stage=None):
    """Run K steps between CUDA events; optionally time one library stage per step."""
    from lagunalab_b200 import _lib
    L = _lib.lib()
    pairs = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = L.lg_launch_count()
    start.record(stream)
    for _ in range(K):
        if profile_stage:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)  # torch creates the event on first record; the library
            e1.record(stream)  # then re-records both around the profiled stage
            L.lg_profile_stage(profile_stage.encode(), e0.cuda_event, e1.cuda_event)
            pairs.append((e0, e1))
        step()
    end.record(stream)
    torch.cuda.synchronize()
    L.lg_profile_stage(None, None, None)
    launches = L.lg_launch_count() - n0
    ms = start.elapsed_time(end) / K
    kernel_ms = statistics.mean(_lib.event_elapsed_ms(a, b) for a, b in pairs) if pairs else None
    return ms, kernel_ms, launches


def run_moe(args, wl, ws, rank):
    from lagunalab_b200 import ep, synth
    T, E, k, H, I, I_sh = (wl[n] for n in ("T", "E", "k", "H", "I", "I_sh"))
    if ws > 1:  # expert parallel over peer memory, T tokens per rank (weak scaling)
        blk = ep.bench_block(E, k, H, I, I_sh, wl["zipf"], wl["scale"])
        g = torch.Generator(device="cuda")
        g.manual_seed(1000 + rank)
        x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
        fwd = ep.PeerExpertParallel(blk, capacity=T)
    else:
        blk, x = synth.moe_block(T, E, k, H, I, I_sh, seed=0, zipf=wl["zipf"],
                                 routed_scaling_factor=wl["scale"])
        fwd = blk
    stream = torch.cuda.current_stream()
    out = fwd(x)
    # routing statistics of the synthetic workload (reported in config)
    inds, _ = blk.route(x)
    counts = torch.bincount(inds.reshape(-1).long(), minlength=E)
    for _ in range(args.warmup):
        fwd(x)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(torch.cuda.current_device())
    time.sleep(0.3)
    clocks.mark(True)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    x_dev = torch.empty_like(x)
    # A decode-size block (config 1) is a few microseconds of kernels: eager ctypes calls
    # would time the host, so one forward is captured in a CUDA graph and replayed per step
    # (the expert-parallel forward passes its epoch as a launch argument and stays eager).
    graphed = ws == 1 and T * k <= 512
    held = {}
    if graphed:
        x_dev.copy_(x)
        g, per_replay, ev = capture(lambda: held.__setitem__("y", fwd(x_dev)), "experts_gateup")
        for _ in range(args.warmup):
            g.replay()
        ms, gu_ms = timed_graph(g, args.steps, stream, ev)
        launches = per_replay * args.steps
    else:
        ms, gu_ms, launches = timed(lambda: fwd(x), args.steps, stream, "experts_gateup")
    barrier(ws)
    # end to end through the module API with host buffers

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        if graphed:
            g.replay()
            o = held["y"]  # the graph's output buffer, rewritten by every replay
        else:
            o = fwd(x_dev)
        out_host.copy_(o, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier(ws)
    e2e_ms, _, _ = timed(e2e_step, args.steps, stream)
    clocks.mark(False)
    barrier(ws)
    ms = max_over_ranks(ms, ws)
    e2e_ms = max_over_ranks(e2e_ms, ws)
    gu_ms = max_over_ranks(gu_ms, ws)
    tokens = T * ws
    return dict(ms=ms, e2e_ms=e2e_ms, kernel_ms=gu_ms, launches=launches, clocks=clocks,
                tokens=tokens, counts=counts, h2d=x.numel() * x.element_size(),
                d2h=out.numel() * out.element_size())


EP_PREFILL = dict(T=32768, E=128, k=8, H=2048, I=1024, I_sh=1024, zipf=True, scale=1.0)


def run_ep_prefill(args, ws, rank):
    """BASELINE config 5 prefill: one MoE layer over 32,768 tokens split evenly over the ranks
    (strong scaling), 128 experts sharded E/N per GPU, Zipf router; the exchange is the
    peer-memory path (lagunalab_b200/ep.py PeerExpertParallel). Rank 0 also times the one-GPU
    block on all 32,768 tokens (the curve's baseline) and checks the gathered expert-parallel
    outputs against it."""
    import torch.distributed as dist
    from lagunalab_b200 import ep
    c = EP_PREFILL
    Tr = c["T"] // ws
    blk = ep.bench_block(c["E"], c["k"], c["H"], c["I"], c["I_sh"], c["zipf"], c["scale"])

    def tokens(r):
        g = torch.Generator(device="cuda")
        g.manual_seed(2000 + r)
        return torch.randn(Tr, c["H"], generator=g, device="cuda").to(torch.bfloat16)

    stream = torch.cuda.current_stream()
    out = dict(tokens=c["T"], experts=c["E"], experts_per_gpu=c["E"] // ws, tokens_per_gpu=Tr,
               n_gpus=ws)
    outs = None
    if ws > 1:
        x = tokens(rank)
        # expert placement balanced on the routing of a separate calibration batch (the same
        # router and Zipf bias, other tokens): greedy, E/N experts per rank
        g = torch.Generator(device="cuda")
        g.manual_seed(3000 + rank)
        xc = torch.randn(Tr, c["H"], generator=g, device="cuda").to(torch.bfloat16)
        cnt = torch.bincount(blk.route(xc)[0].reshape(-1).long(), minlength=c["E"])
        dist.all_reduce(cnt)
        placement = ep.balanced_placement(cnt.tolist(), ws)
        pe = ep.PeerExpertParallel(blk, capacity=Tr, placement=placement)
        # picks per owner on the measured batch under that placement
        own = torch.empty(c["E"], dtype=torch.long, device="cuda")
        for d, p in enumerate(placement):
            own[torch.tensor(p, device="cuda")] = d
        mine = torch.bincount(own[blk.route(x)[0].reshape(-1).long()], minlength=ws)
        dist.all_reduce(mine)
        loads = mine.tolist()
        for _ in range(args.warmup):
            pe(x)
        torch.cuda.synchronize()
        barrier(ws)
        ms, _, launches = timed(lambda: pe(x), args.steps, stream)
        ms = max_over_ranks(ms, ws)
        y = pe(x)
        torch.cuda.synchronize()
        status = int(max_over_ranks(float(pe.status()), ws))
        outs = [torch.empty_like(y) for _ in range(ws)]
        dist.all_gather(outs, y)
        pe.close()
        out.update(ms_per_step=ms, tokens_per_s=c["T"] / (ms * 1e-3), status=status,
                   gpu_launches_per_step=launches // max(1, args.steps),
                   exchange="NVLink peer stores issued by the dispatch kernel and the expert "
                            "down-product epilogue; epoch flags with bounded waits; no collective",
                   placement="balanced (greedy, E/N experts per rank) on the picks of a separate "
                             "calibration batch",
                   picks_per_owner=loads,
                   owner_max_over_mean=max(loads) * len(loads) / max(1, sum(loads)))
    if rank == 0:
        xa = torch.cat([tokens(r) for r in range(ws)])
        for _ in range(args.warmup):
            blk(xa)
        torch.cuda.synchronize()
        ms1, _, _ = timed(lambda: blk(xa), args.steps, stream)
        out.update(one_gpu_ms=ms1, one_gpu_tokens_per_s=c["T"] / (ms1 * 1e-3))
        if outs is not None:
            ref = blk(xa).float()
            got = torch.cat(outs).float()
            out.update(speedup=ms1 / out["ms_per_step"],
                       efficiency=ms1 / (out["ms_per_step"] * ws),
                       identical_to_one_gpu=bool(torch.equal(got, ref)),
                       max_rel_err=float((got - ref).abs().max() / ref.abs().max()),
                       cosine=float(torch.nn.functional.cosine_similarity(
                           got.reshape(-1), ref.reshape(-1), dim=0)))
    del blk
    torch.cuda.empty_cache()
    barrier(ws)
    return out


DECODE_STREAMS = dict(B=64, ctx=8192, experts=128, seed=1, steps=8, warmup=3)


def _stream_model(c):
    from lagunalab_b200 import synth
    wl = dict(WORKLOADS["decode"], experts=c["experts"], seed=c["seed"])
    _, model = decode_model(wl)
    synth.zipf_router(model, seed=c["seed"])
    return model


def run_decode_streams(args, ws, rank):
    """BASELINE config 5's batched decode: the unpruned 128-expert decoder (config 2's MoE shape
    in the config-3 decoder; Zipf(1.1)-skewed router), 64 concurrent streams at an 8,192-token
    context each, one greedy token per stream per step, each step one CUDA-graph replay. The
    streams are split evenly over the ranks (strong scaling: 64 streams in all); with N > 1
    every MoE layer runs expert parallel (E/N experts per rank; dispatch and return are NVLink
    peer stores issued by the kernels, with device-held epochs so the exchanges replay with the
    graph). Each stream's cache holds synthetic K/V rows for its 8,192 context positions (seeded
    N(0, 1)) instead of a prefill: a decode step reads the same bytes either way. Rank 0 also
    times all 64 streams on its own GPU with every expert local (the one-GPU baseline)."""
    import torch.distributed as dist
    from lagunalab_b200 import _lib, ep, laguna, synth
    c = DECODE_STREAMS
    B, ctx = c["B"], c["ctx"]
    Br = B // ws
    K, Wm = c["steps"], c["warmup"]
    cap = (ctx + K + Wm + 2 + 255) // 256 * 256
    model = _stream_model(c)
    stream = torch.cuda.current_stream()

    def streams(first, n):
        cache = model.make_stream_cache(n, cap)
        synth.fill_stream_cache(cache, ctx, first_stream=first, seed=c["seed"])
        g = torch.Generator().manual_seed(c["seed"] + 99)
        ids = torch.randint(0, model.args.vocab_size, (B,), generator=g)[first:first + n]
        return cache, ids.to(torch.int32).cuda(), torch.full((n,), ctx, dtype=torch.int32,
                                                              device="cuda")

    def time_graph(g, profiled=False):
        for _ in range(Wm):
            g.step()
        torch.cuda.synchronize()
        if profiled:  # an NVTX range a profiler can select (ncu --nvtx-include decode_streams/)
            torch.cuda.nvtx.range_push("decode_streams")
        try:
            return timed_graph(g.graph, K, stream)[0]
        finally:
            if profiled:
                torch.cuda.nvtx.range_pop()

    out = dict(streams=B, context=ctx, experts=c["experts"], n_gpus=ws, streams_per_gpu=Br,
               kv="bf16", steps=K,
               data="synthetic K/V context rows (seeded N(0,1)); random-init 4-bit weights")
    pes = []
    if ws > 1:
        moe = []
        for L in model.layers:
            if isinstance(L.mlp, laguna.SparseMoeBlock):
                # the owners' product path is fixed so every rank takes the same one
                pes.append(ep.PeerExpertParallel(L.mlp, capacity=Br, device_epoch=True,
                                                 expert_path=_lib.LG_PATH_GEMV))
                moe.append(pes[-1])
            else:
                moe.append(None)
        cache, tok, pos = streams(rank * Br, Br)
        g = laguna.StreamDecodeGraph(model, cache, tok, pos, moe=moe)
        barrier(ws)
        ms = max_over_ranks(time_graph(g), ws)
        torch.cuda.synchronize()
        status = int(max_over_ranks(float(max(p.status() for p in pes)), ws))
        out.update(ms_per_step=ms, tokens_per_s=B / (ms * 1e-3), status=status,
                   exchange="NVLink peer stores issued by the dispatch kernel and the expert "
                            "down-product epilogue; device-held epochs; no collective")
        del g, cache
        torch.cuda.empty_cache()
    if rank == 0:
        cache, tok, pos = streams(0, B)
        # the library records an event pair around the attention launches while the step is
        # captured; the pair ends up around the step's last one
        L = _lib.lib()
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        ev[1].record()
        L.lg_profile_stage(b"bf16_decode", ev[0].cuda_event, ev[1].cuda_event)
        try:
            g1 = laguna.StreamDecodeGraph(model, cache, tok, pos)
        finally:
            L.lg_profile_stage(None, None, None)
        ms1 = time_graph(g1, profiled=ws == 1)
        at = []
        for _ in range(3):
            g1.step()
            torch.cuda.synchronize()
            at.append(_lib.event_elapsed_ms(ev[0], ev[1]))
        at_ms = statistics.median(at)
        nbytes = B * model.args.num_key_value_heads * (ctx + K + Wm + 4) * 512
        pk, pk_kind = peaks()
        out.update(one_gpu_ms=ms1, one_gpu_tokens_per_s=B / (ms1 * 1e-3),
                   attention={"kernel": "bf16_decode_kernel", "us": at_ms * 1e3,
                              "achieved_gbs": nbytes / (at_ms * 1e-3) / 1e9,
                              "frac": nbytes / (at_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                              "peak_source": pk_kind,
                              "algorithmic": "streams x kv heads x keys x 512 B (bf16 K and V "
                                             "rows), at the timed steps' context"})
        if ws > 1:
            out.update(speedup=ms1 / out["ms_per_step"],
                       efficiency=ms1 / (out["ms_per_step"] * ws))
        else:
            out.update(ms_per_step=ms1, tokens_per_s=B / (ms1 * 1e-3))
        del g1, cache
    barrier(ws)
    for p in pes:
        p.close()
    del model, pes
    torch.cuda.empty_cache()
    barrier(ws)
    return out


def capture(fn, profile_stage=None):
    """Capture fn() into a CUDA graph after one eager call on a side stream. With
    profile_stage, the library records a pair of external event nodes around that stage, so
    every replay re-times the stage's last launch in the graph."""
    from lagunalab_b200 import _lib
    L = _lib.lib()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    ev = None
    if profile_stage:
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        ev[1].record()
        L.lg_profile_stage(profile_stage.encode(), ev[0].cuda_event, ev[1].cuda_event)
    g = torch.cuda.CUDAGraph()
    n0 = L.lg_launch_count()
    try:
        with torch.cuda.graph(g):
            fn()
    finally:
        L.lg_profile_stage(None, None, None)
    return g, L.lg_launch_count() - n0, ev


def timed_graph(g, K, stream, ev=None, samples=10):
    """K back-to-back replays between CUDA events; then a few synchronised replays that read
    the profiled stage's event pair."""
    from lagunalab_b200 import _lib
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(K):
        g.replay()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / K
    kernel_ms = None
    if ev is not None:
        t = []
        for _ in range(samples):
            g.replay()
            torch.cuda.synchronize()
            t.append(_lib.event_elapsed_ms(ev[0], ev[1]))
        kernel_ms = statistics.median(t)
    return ms, kernel_ms


def run_q8(args, wl, ws, rank):
    """40 layers of q8 decode attention, each call through the public API, captured once into
    a CUDA graph and replayed per step (the per-call host cost of a Python ctypes call would
    otherwise exceed the kernel's ~15 us)."""
    from lagunalab_b200 import ops, synth
    L, n, B, Hq, Hkv = (wl[k] for k in ("L", "n", "B", "Hq", "Hkv"))
    layers = synth.q8_layers(L, n, B, Hq, Hkv, seed=rank)
    scale = 128 ** -0.5
    outs = [torch.empty_like(q) for q, _, _ in layers]

    def step():
        for (q, kt, vt), o in zip(layers, outs):
            ops.q8_decode_attention(q, kt, vt, n, scale, out=o)

    stream = torch.cuda.current_stream()
    g, per_replay, _ = capture(step)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(torch.cuda.current_device())
    time.sleep(0.3)
    clocks.mark(True)
    ms, _ = timed_graph(g, args.steps, stream)
    # the step is L launches of the one kernel back to back: its average launch duration is
    # the step time / L (gaps between launches included, so this understates the kernel)
    k_ms = ms / L
    # end to end: every step uploads all layers' q from pinned host memory in one copy, runs
    # the 40 public-API calls and reads every output back in one copy
    q_host = torch.stack([q for q, _, _ in layers]).cpu().pin_memory()
    q_dev = torch.empty_like(q_host, device="cuda")
    o_dev = torch.empty_like(q_dev)
    o_host = torch.empty_like(q_host).pin_memory()

    def e2e_body():
        for i, (_, kt, vt) in enumerate(layers):
            ops.q8_decode_attention(q_dev[i], kt, vt, n, scale, out=o_dev[i])

    # the copies are stream operations around the kernel-only graph (copy nodes inside a graph
    # cost its kernels their programmatic-launch edges)
    ge, _, _ = capture(e2e_body)

    class _E2E:
        @staticmethod
        def replay():
            q_dev.copy_(q_host, non_blocking=True)
            ge.replay()
            o_host.copy_(o_dev, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        _E2E.replay()
    torch.cuda.synchronize()
    e2e_ms, _ = timed_graph(_E2E, args.steps, stream)
    clocks.mark(False)
    ms = max_over_ranks(ms, ws)
    e2e_ms = max_over_ranks(e2e_ms, ws)
    del g, ge
    return dict(ms=ms, e2e_ms=e2e_ms, kernel_ms=k_ms, launches=per_replay * args.steps,
                clocks=clocks, bytes=synth.q8_bytes_per_layer(n, B, Hkv) * L * ws,
                h2d=q_host.numel() * q_host.element_size(),
                d2h=o_host.numel() * o_host.element_size(), graph=True)


def decode_model(wl):
    from lagunalab_b200 import synth
    a = synth.decoder_args(vocab=wl["vocab"], hidden=wl["hidden"], layers=wl["layers"],
                           heads=wl["heads"], kv_heads=wl["kv_heads"], head_dim=wl["head_dim"],
                           experts=wl["experts"], top_k=wl["top_k"], moe_inter=wl["moe_inter"],
                           shared_inter=wl["shared_inter"], dense_inter=wl["dense_inter"],
                           rope_theta=wl["rope_theta"])
    return a, synth.decoder(a, seed=wl["seed"])


def decode_bytes_per_token(model, ctx, kv="bf16"):
    """HBM bytes one decode step must read: every dense weight of the step (attention,
    router, shared expert, dense layer 0, lm_head), the top-k routed experts of each MoE
    layer, one embedding row, and the K/V rows of ctx keys per layer (bf16: 2 B per element;
    8-bit g64: 1 B per element plus a bf16 scale and bias per 64)."""
    from lagunalab_b200 import laguna
    nb = lambda m: sum(t.numel() * t.element_size() for t in m.mat)
    a = model.args
    row = a.head_dim * 2 if kv == "bf16" else a.head_dim + (a.head_dim // 64) * 4
    total = sum(nb(x) for x in (model.lm_head,)) + nb(model.model.embed_tokens) // a.vocab_size
    for L in model.layers:
        at = L.self_attn
        total += nb(at._qkvg) + nb(at.o_proj)
        total += 2 * a.num_key_value_heads * ctx * row
        m = L.mlp
        if isinstance(m, laguna.MLP):
            total += sum(nb(p) for p in (m.gate_proj, m.up_proj, m.down_proj))
        else:
            total += nb(m.gate) + sum(nb(p) for p in (m.shared_expert.gate_proj,
                                                       m.shared_expert.up_proj,
                                                       m.shared_expert.down_proj))
            per_expert = sum(nb(p) for p in (m.switch_mlp.gate_proj, m.switch_mlp.up_proj,
                                             m.switch_mlp.down_proj)) // a.num_experts
            total += a.num_experts_per_tok * per_expert
    return total


def run_decode(args, wl, ws, rank):
    """prefill wl["prefill"] uniform-random ids (seed 1), then greedy decode
    one token per step, each step one replay of a CUDA graph of the whole model (token id and
    cache position stay on the device). kv "q8": the 8-bit quantized cache."""
    from lagunalab_b200 import laguna, ops
    margs, model = decode_model(wl)
    V = margs.vocab_size
    g = torch.Generator().manual_seed(wl["seed"])
    prompt = torch.randint(0, V, (wl["prefill"],), generator=g).to(torch.int32).cuda()
    n_steps = 1 + args.warmup + args.steps + 1 + max(1, args.warmup) + args.steps + 2 + 12
    cap = (wl["prefill"] + n_steps + 255) // 256 * 256
    if wl.get("kv") == "q8":
        from lagunalab_b200 import cache as qcache
        cache = qcache.make_quantized_cache(model, fused_decode=True, capacity=cap)
    else:
        cache = model.make_cache(capacity=cap)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    logits = model.last_logits(prompt.view(1, -1), cache)
    e1.record(stream)
    tok = ops.argmax(logits.view(1, -1))
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    n0 = _lib_launches()
    dg = laguna.DecodeGraph(model, cache, tok)  # one eager step, then the capture
    per_replay = _lib_launches() - n0
    per_replay //= 2  # the eager step and the capture each issue the step's launches once
    for _ in range(args.warmup):
        dg.step()
    torch.cuda.synchronize()
    ctx0 = dg.position()
    clocks = ClockSampler(torch.cuda.current_device())
    time.sleep(0.3)
    clocks.mark(True)
    barrier(ws)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("decode_step")
    ms, _ = timed_graph(dg.graph, args.steps, stream)
    torch.cuda.nvtx.range_pop()
    barrier(ws)
    dg.steps += args.steps
    ctx1 = dg.position()
    # end to end: every step uploads the input token from pinned host memory, runs the step
    # and reads the generated token back to the host, which feeds it to the next step. The
    # copies are stream operations around the step's kernel-only graph: copy nodes inside the
    # graph cost its kernels their programmatic-launch edges (~0.2 ms a step).
    tok_in = torch.empty(1, dtype=torch.int32).pin_memory()
    tok_out = torch.empty(1, dtype=torch.int32).pin_memory()
    tok_out.copy_(dg.tok.cpu())
    t_in, t_out = tok_in.numpy(), tok_out.numpy()

    def e2e_step():
        t_in[0] = t_out[0]
        dg.tok.copy_(tok_in, non_blocking=True)
        dg.graph.replay()
        tok_out.copy_(dg.tok, non_blocking=True)
        torch.cuda.synchronize()

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier(ws)
    t0 = time.perf_counter()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = s0.elapsed_time(s1) / args.steps
    clocks.mark(False)
    # the dominant kernel, timed live: a graph of the same step in which the library records
    # an event pair around that stage's launches (the pair ends up around the step's last one)
    from lagunalab_b200 import _lib
    L = _lib.lib()
    stage = "q8_decode" if wl.get("kv") == "q8" else "moe_decode"
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev[0].record()
    ev[1].record()
    L.lg_profile_stage(stage.encode(), ev[0].cuda_event, ev[1].cuda_event)
    prev = L.lg_set_pdl(1)
    gk = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(gk):
            dg._body()
    finally:
        L.lg_set_pdl(prev)
        L.lg_profile_stage(None, None, None)
    kt = []
    for _ in range(12):
        gk.replay()
        torch.cuda.synchronize()
        kt.append(_lib.event_elapsed_ms(ev[0], ev[1]))
    kernel_ms = statistics.median(kt[2:])
    ctx_k = dg.position()
    # N GPUs run N independent replicas of the bs1 decode: the slowest rank sets the time
    ms, e2e_ms, kernel_ms = (max_over_ranks(v, ws) for v in (ms, e2e_ms, kernel_ms))
    ctx = (ctx0 + ctx1) / 2
    del gk
    a_ = model.args
    if stage == "q8_decode":
        kbytes = ctx_k * a_.num_key_value_heads * (2 * (a_.head_dim + 4 * (a_.head_dim // 64)))
    else:
        nb = lambda m: sum(t.numel() * t.element_size() for t in m.mat)
        m = next(l.mlp for l in model.layers if hasattr(l.mlp, "switch_mlp"))
        per_expert = sum(nb(p) for p in (m.switch_mlp.gate_proj, m.switch_mlp.up_proj,
                                         m.switch_mlp.down_proj)) // a_.num_experts
        kbytes = a_.num_experts_per_tok * per_expert + sum(
            nb(p) for p in (m.shared_expert.gate_proj, m.shared_expert.up_proj,
                            m.shared_expert.down_proj))
    return dict(ms=ms, e2e_ms=e2e_ms, launches=per_replay * args.steps, clocks=clocks,
                kernel=stage, kernel_ms=kernel_ms, kernel_bytes=kbytes, kernel_ctx=ctx_k,
                bytes=decode_bytes_per_token(model, ctx, wl.get("kv", "bf16")), ctx=(ctx0, ctx1),
                prefill_ms=prefill_ms,
                h2d=4, d2h=4)


def _lib_launches():
    from lagunalab_b200 import _lib
    return _lib.lib().lg_launch_count()


# ----------------------------------------------------------------------------------------
# CPU baseline (the oracle restatement timed on the host cores; rank 0 only)
# ----------------------------------------------------------------------------------------

def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_moe(wl, steps, warmup, sample_tokens=256):
    """The oracle's MoE block (pre-dequantized fp32 weights) on a sample of the workload."""
    from oracle import moe_ref
    from lagunalab_b200 import synth
    T, E, k, H, I, I_sh = (wl[n] for n in ("T", "E", "k", "H", "I", "I_sh"))
    # weights drawn and kept on the CPU (the library is never loaded on this leg)
    g = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02
    wg, wu, wd = r(E, I, H), r(E, I, H), r(E, H, I)
    sh = (r(I_sh, H), r(I_sh, H), r(H, I_sh))
    router = r(E, H)
    bias = synth.zipf_bias(E, 0, device="cpu") if wl["zipf"] else torch.zeros(E)
    xs = torch.randn(sample_tokens, H, generator=g).to(torch.bfloat16)
    nt = cpu_threads()
    torch.set_num_threads(nt)

    def step():
        inds, w, *_ = moe_ref.route(xs, router, bias, k)
        y = moe_ref.switch_glu_deq(xs, inds, wg, wu, wd)
        return moe_ref.combine(y, w, wl["scale"], moe_ref.mlp_deq(xs, *sh))

    for _ in range(warmup):
        step()
    t = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        t.append(time.perf_counter() - t0)
    sec = statistics.median(t)
    return dict(value=sample_tokens / sec, unit="tokens/s", cores=nt, kind="port",
                sample=f"{sample_tokens} of the {T} tokens per step, same weights and routing "
                       f"(oracle restatement, weights pre-dequantized to fp32)")


def cpu_q8(wl, steps, warmup, sample_layers=1):
    from oracle import attn_ref
    from lagunalab_b200 import synth
    n, B, Hq, Hkv = (wl[k] for k in ("n", "B", "Hq", "Hkv"))
    # cache rows quantized on the CPU (the library is never loaded on this leg)
    layers = []
    for _ in range(sample_layers):
        g = torch.Generator().manual_seed(0)
        mk = lambda: tuple(
            torch.from_numpy(a.view("int32") if a.dtype.kind == "u" and a.itemsize == 4
                             else a.view("int16")) for a in
            attn_ref.quantize_rows(torch.randn(B, Hkv, n, 128, generator=g).numpy(), 64, 8))
        kt, vt = mk(), mk()
        kt = (kt[0], kt[1].view(torch.bfloat16), kt[2].view(torch.bfloat16))
        vt = (vt[0], vt[1].view(torch.bfloat16), vt[2].view(torch.bfloat16))
        layers.append((torch.randn(B, Hq, 1, 128, generator=g).to(torch.bfloat16), kt, vt))
    nt = cpu_threads()
    torch.set_num_threads(nt)

    def step():
        for q, kt, vt in layers:
            attn_ref.q8_decode_attention_ref(q, kt, vt, n, 128 ** -0.5)

    for _ in range(warmup):
        step()
    t = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        t.append(time.perf_counter() - t0)
    sec = statistics.median(t)
    gbs = synth.q8_bytes_per_layer(n, B, Hkv) * sample_layers / sec / 1e9
    return dict(value=gbs, unit="GB/s", cores=nt, kind="port",
                sample=f"{sample_layers} of the {wl['L']} layers per step at {n} keys "
                       f"(oracle restatement: dequantize + fp32 softmax)")


def _oracle_quantize(t, bits):
    """The oracle's quantizer in threads over row blocks -> torch (int32, bf16, bf16)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle import attn_ref
    x = t.reshape(-1, t.shape[-1]).numpy()
    blocks = [r for r in np.array_split(np.arange(x.shape[0]), cpu_threads()) if len(r)]
    with ThreadPoolExecutor(len(blocks)) as ex:
        parts = list(ex.map(lambda r: attn_ref.quantize_rows(x[r[0]:r[-1] + 1], 64, bits),
                            blocks))
    cat = lambda j: np.concatenate([q[j] for q in parts]).reshape(*t.shape[:-1], -1)
    return (torch.from_numpy(cat(0).view(np.int32)),
            torch.from_numpy(cat(1).view(np.int16)).view(torch.bfloat16),
            torch.from_numpy(cat(2).view(np.int16)).view(torch.bfloat16))


class _PackedKV:
    """The 8-bit (or bf16) KV cache as the reference's CPU path keeps it: preallocated packed
    rows; an append quantizes the new rows into place, and a step attends over all rows
    dequantized to bf16 (DequantKVCache without the fused Metal kernel, which the CPU backend
    cannot run: laguna_mlx/cache.py:89-100). One buffer serves every layer (each layer costs
    the same; the rows' values do not change the work)."""

    def __init__(self, kv, rows, cap, Hkv, D):
        from oracle import attn_ref, moe_ref
        self.kv, self.offset = kv, rows
        from lagunalab_b200 import synth
        k, v = synth.kv_rows(0, cap, Hkv, D, seed=0, device="cpu")
        if kv == "q8":
            self.k = _oracle_quantize(k.float(), 8)
            self.v = _oracle_quantize(v.float(), 8)
        else:
            self.k, self.v = k, v
        self._attn_ref, self._moe_ref = attn_ref, moe_ref

    def _rows(self, t, n):
        if self.kv != "q8":
            return t[:, :n].float()
        q, s, b = t
        return self._moe_ref.dequantize(q[:, :n], s[:, :n], b[:, :n], 64, 8).to(
            torch.bfloat16).float()

    def update(self, i, k, v):
        T = k.shape[1]
        n0 = self.offset
        if self.kv == "q8":
            for dst, x in ((self.k, k), (self.v, v)):
                q, s_, b_ = _oracle_quantize(x.contiguous(), 8)
                dst[0][:, n0:n0 + T], dst[1][:, n0:n0 + T], dst[2][:, n0:n0 + T] = q, s_, b_
        else:
            self.k[:, n0:n0 + T] = k.to(torch.bfloat16)
            self.v[:, n0:n0 + T] = v.to(torch.bfloat16)
        return self._rows(self.k, n0 + T), self._rows(self.v, n0 + T)


def cpu_decode(wl, steps, warmup, budget_s=60.0):
    """One greedy decode token of the workload's model through the oracle's restatement of the
    reference's CPU path (laguna_mlx/laguna.py:75-206 with the KV cache of cache.py:89-100),
    on the host cores, with weights built on the CPU (the counter-based generator and the
    oracle's quantizer: the library is never loaded). A token runs all layers — the dense
    layer 0, then the MoE layer weights for every one of the other layers (one MoE layer is
    built and reused: each costs the same) — and the lm_head, at the workload's context over a
    preallocated cache in the workload's KV format. As many whole tokens are timed as fit in
    ``budget_s`` (at least one, at most ``steps``), after ``warmup`` untimed MoE layers."""
    from oracle import model_ref
    from lagunalab_b200 import synth
    nt = cpu_threads()
    torch.set_num_threads(nt)
    a = synth.decoder_args(vocab=wl["vocab"], hidden=wl["hidden"], layers=wl["layers"],
                           heads=wl["heads"], kv_heads=wl["kv_heads"], head_dim=wl["head_dim"],
                           experts=wl["experts"], top_k=wl["top_k"], moe_inter=wl["moe_inter"],
                           shared_inter=wl["shared_inter"], dense_inter=wl["dense_inter"],
                           rope_theta=wl["rope_theta"])
    keep = ("model.embed_tokens", "model.norm", "lm_head", "model.layers.0.", "model.layers.1.")
    items = synth.decoder_tensors(a, seed=wl["seed"], device="cpu",
                                  want=lambda n: n.startswith(keep))
    W = model_ref.weights_from_named(items, 2, _oracle_quantize)
    W["layers"] = [W["layers"][0]] + [W["layers"][1]] * (a.num_hidden_layers - 1)
    oa = synth.oracle_args(a)
    ctx = wl["prefill"]
    cap = ctx + steps + warmup + 2
    cache = _PackedKV(wl.get("kv", "bf16"), ctx, cap, a.num_key_value_heads, a.head_dim)
    tok = [7]
    one = dict(W, layers=W["layers"][1:2])
    for _ in range(warmup):  # untimed: one MoE layer
        model_ref.forward(one, oa, tok, cache)
        cache.offset -= 1
    times = []
    t_all = time.perf_counter()
    while len(times) < max(1, steps):
        t0 = time.perf_counter()
        logits = model_ref.forward(W, oa, tok, cache)
        tok = [int(torch.argmax(logits[-1]))]
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    sec = statistics.median(times)
    return dict(value=1.0 / sec, unit="tokens/s", cores=nt, kind="port",
                sample=f"{len(times)} whole decode tokens timed ({a.num_hidden_layers} layers + "
                       f"lm_head each; median) at context {ctx} with a {wl.get('kv', 'bf16')} "
                       f"KV cache (oracle restatement of the reference's CPU path; one MoE "
                       f"layer's weights serve all MoE layers and one cache serves all layers)")


# ----------------------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="decode_q8")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep", action="store_true",
                    help="skip the config-5 expert-parallel prefill measurement")
    ap.add_argument("--no-streams", action="store_true",
                    help="skip the config-5 batched decode measurement (64 streams x 8k)")
    ap.add_argument("--layers", type=int, default=None,
                    help="q8_decode only: layers per step (default: the config's 40; fewer "
                         "for small profiling runs)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    wl = dict(WORKLOADS[args.workload])
    if args.layers and args.workload == "q8_decode":
        wl["L"] = args.layers
    if args.impl == "reference":
        # the reference arm runs on rank 0's host cores alone: other ranks exit at once (no
        # process group, nothing spinning on a core), and rank 0 never loads the library
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        if int(os.environ.get("RANK", "0")) != 0:
            return
        if args.workload == "q8_decode":
            ref = cpu_q8(wl, args.steps, args.warmup)
        elif args.workload in DECODE_WORKLOADS:
            ref = cpu_decode(wl, args.steps, 1)
        else:
            ref = cpu_moe(wl, args.steps, args.warmup)
        metric, unit = metric_unit(args.workload)
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": ref["value"], "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": config(args, wl, ws),
            "cpu_baseline": {"value": ref["value"], "unit": unit, "cores": ref["cores"],
                             "kind": ref["kind"], "sample": ref["sample"]},
            "e2e": {"value": ref["value"], "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    ws, rank, local = dist_setup()

    pk, pk_kind = peaks()
    decode_info = None
    if args.workload in DECODE_WORKLOADS:
        r = run_decode(args, wl, ws, rank)
        value = ws * 1000.0 / r["ms"]  # every replica decodes one token per step
        e2e = ws * 1000.0 / r["e2e_ms"]
        step_gbs = r["bytes"] / (r["ms"] * 1e-3) / 1e9
        achieved = r["kernel_bytes"] / (r["kernel_ms"] * 1e-3) / 1e9
        if r["kernel"] == "q8_decode":
            prof, name = "q8_decode_kernel_config4", "q8_decode_kernel"
            alg = (f"{r['kernel_bytes']:.0f} B per launch ({r['kernel_ctx']} keys x 4 kv heads x "
                   f"272 B: 8-bit K and V rows with their bf16 scales and biases)")
        else:
            prof, name = "moe_decode_config3", "moe_dec_gateup_kernel + moe_dec_down_kernel"
            alg = (f"{r['kernel_bytes']:.0f} B per call (top-k picked experts + shared expert, "
                   f"gate/up/down at 0.5625 B per weight)")
        roof = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                "traffic": profile_traffic(prof), "peak_source": pk_kind, "algorithmic": alg,
                "duration": "CUDA events around the stage's last launch in a replayed step graph",
                "traffic_source": f"profiles/{prof}.md (ncu, one launch)",
                "step": {"achieved": step_gbs, "frac": step_gbs / pk["hbm_gbs"],
                         "algorithmic": f"{r['bytes']:.0f} B per token (weights read by one "
                                        f"step, top-k experts, {wl['kv']} K/V at mean context "
                                        f"{sum(r['ctx']) / 2:.0f})",
                         "duration": "graph step time (one replay per token)"}}
        decode_info = {"prefill_ms": r["prefill_ms"], "context": list(r["ctx"])}
        dtype = "bf16"
    elif args.workload == "q8_decode":
        r = run_q8(args, wl, ws, rank)
        value = r["bytes"] / (r["ms"] * 1e-3) / 1e9
        e2e = r["bytes"] / (r["e2e_ms"] * 1e-3) / 1e9
        per_launch = r["bytes"] / wl["L"] / ws
        achieved = per_launch / (r["kernel_ms"] * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "q8_decode_kernel", "achieved": achieved,
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                "traffic": profile_traffic("q8_decode_kernel_config4"), "peak_source": pk_kind,
                "algorithmic": f"{per_launch:.0f} B per launch (n x Hkv x 272 B)",
                "duration": "graph step time / launches per step (inter-launch gaps included)",
                "traffic_source": "profiles/q8_decode_kernel_config4.md (ncu, one launch)"}
        dtype = "u8"
    else:
        r = run_moe(args, wl, ws, rank)
        value = r["tokens"] / (r["ms"] * 1e-3)
        e2e = r["tokens"] / (r["e2e_ms"] * 1e-3)
        from lagunalab_b200 import synth
        fl = synth.gateup_flops(wl["T"], wl["k"], wl["H"], wl["I"], wl["I_sh"])
        if ws > 1:
            fl = None
        achieved = fl / (r["kernel_ms"] * 1e-3) / 1e12 if fl else None
        peak = pk["bf16_tflops"]
        roof = {"bound": "tensor", "kernel": "experts_gateup", "achieved": achieved,
                "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak if achieved else None,
                "traffic": profile_traffic("moe_tc_gateup_config2"),
                "peak_source": pk_kind,
                "algorithmic": "2 * 2I * H FLOP per routed pick and shared row",
                "traffic_source": "profiles/moe_tc_gateup_config2.md (ncu, one launch)"}
        c = r["counts"]
        wl = dict(wl, max_count=int(c.max()), min_count=int(c.min()),
                  distinct=int((c > 0).sum()))
        dtype = "bf16"
    metric, unit = metric_unit(args.workload)
    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": config(args, wl, ws),
        "e2e": {"value": e2e, "unit": unit, "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": r["d2h"], "ms_per_step": r["e2e_ms"]},
        "roofline": roof,
        "gpu_launches": r["launches"] * (ws if args.workload in DECODE_WORKLOADS else 1),
        "clocks": r["clocks"].result(),
    }
    if decode_info:
        line["decode"] = decode_info
    if not args.no_ep:
        line["ep_prefill"] = run_ep_prefill(args, ws, rank)
    if not args.no_streams:
        line["decode_streams"] = run_decode_streams(args, ws, rank)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cb = (cpu_q8(wl, 3, 1) if args.workload == "q8_decode" else
              cpu_decode(wl, 2, 1, budget_s=45.0) if args.workload in DECODE_WORKLOADS else cpu_moe(wl, 5, 1))
        line["cpu_baseline"] = cb
    if rank == 0:
        print(json.dumps(line), flush=True)
    finish(ws)


def metric_unit(workload):
    if workload == "decode":
        return "bs1 decode tok/s @8k ctx (config 3, bf16 KV)", "tokens/s"
    if workload == "decode_q8":
        return "bs1 decode tok/s @82k ctx (config 3 model, 8-bit KV)", "tokens/s"
    if workload == "q8_decode":
        return "q8 decode attention HBM GB/s (40 layers @82,671 ctx)", "GB/s"
    if workload == "moe_decode":
        return "MoE-layer tokens/s (T=16)", "tokens/s"
    return "MoE-layer tokens/s", "tokens/s"


def config(args, wl, ws):
    c = {"workload": args.workload, **{k: v for k, v in wl.items()}}
    c["l2"] = "inputs larger than L2 (126 MB): weights/KV streamed from HBM each step"
    if args.workload in DECODE_WORKLOADS:
        c["launch"] = ("prefill through the module API, then one CUDA-graph replay per decoded "
                       "token (token id and cache position kept on the device); e2e feeds each "
                       "token through pinned host memory and synchronises every step")
        c["weights"] = "random-init, 4-bit g64 linears and embedding, 8-bit router"
    if args.workload == "q8_decode":
        c["launch"] = ("the step's 40 public-API calls captured once in a CUDA graph and "
                       "replayed per step; e2e adds each step's q upload from pinned host "
                       "memory before the replay and the output read-back after it")
    c["parallelism"] = f"ep{ws}" if ws > 1 and args.workload not in ("q8_decode", *DECODE_WORKLOADS) else \
        (f"replicas{ws}" if ws > 1 else "single")
    return c


def finish(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
