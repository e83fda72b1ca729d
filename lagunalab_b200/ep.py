"""Expert parallelism for the MoE block over the GPUs of one node (the
reference runs on one device and has no counterpart).

Rank r of W owns the contiguous experts [r*E/W, (r+1)*E/W); the router and the shared expert
are replicated and every rank routes its own tokens. One forward, on every rank alike:

1. route locally (the router kernel): inds [T, k], w [T, k];
2. dispatch: each token with at least one pick owned by rank d is sent to d once, into slot
   s of d's receive rows for this source (slots in token order), with its k expert ids local
   to d (-1 for picks owned elsewhere), its k routing weights and its token index;
3. the owner runs its experts over the received rows (the grouped kernels) and returns, for
   every pick, bf16(bf16(y) * w) into the source's combine row (token * k + j);
4. combine at the source in pick order: bf16(bf16(bf16(sum_j rows) * scale) + shared(x)),
   the arithmetic of the one-GPU block, so the outputs are bit-identical to it.

``PeerExpertParallel`` is the B200 path: the exchanges are NVLink peer stores from inside the
kernels (``csrc/ep.cu``) into per-rank arenas mapped with CUDA IPC, synchronised by epoch flags
with bounded waits; no host synchronisation and no collective in the data path.
``CollectiveExpertParallel`` runs the same data flow with fixed-capacity torch all-to-alls
(``capacity`` rows per rank pair, so no host read of counts) and injectable compute, so the
control flow is tested on gloo CPU ranks with the oracle's arithmetic.
"""
import ctypes

import torch
import torch.distributed as dist


def _bf(t):
    return t.to(torch.bfloat16).to(torch.float32)


def plan_slots(inds, El, W):
    """Per (token, destination): the token's slot in that destination's receive rows, or -1
    when none of its picks is owned there (slots in token order). inds [T, k] -> [T, W]."""
    owner = torch.where(inds >= 0, torch.div(inds, El, rounding_mode="floor"), -1)
    has = torch.stack([(owner == d).any(-1) for d in range(W)], dim=-1)  # [T, W]
    slot = torch.cumsum(has.to(torch.int64), 0) - 1
    return torch.where(has, slot, torch.full_like(slot, -1))


class CollectiveExpertParallel:
    """The expert-parallel data flow with fixed-capacity torch all-to-alls (gloo or NCCL).

    ``route_fn(x) -> (inds [T, k], w [T, k])``; ``expert_fn(rows [R, H], lid [R, k]) -> y
    [R, k, H]`` (the local experts' per-pick outputs, ignored where lid < 0); ``shared_fn(x)
    -> [T, H]``. ``capacity`` bounds the tokens per rank and forward (the same on all ranks)."""

    def __init__(self, E, k, routed_scaling_factor, route_fn, expert_fn, shared_fn=None,
                 capacity=4096, group=None):
        self.group = group
        self.W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.W:
            raise ValueError(f"{E} experts do not split evenly over {self.W} ranks")
        self.E, self.k, self.El, self.cap = E, k, E // self.W, capacity
        self.scale = routed_scaling_factor
        self.route_fn, self.expert_fn, self.shared_fn = route_fn, expert_fn, shared_fn

    def _a2a(self, t):
        out = torch.empty_like(t)
        dist.all_to_all_single(out, t.contiguous(), group=self.group)
        return out

    def __call__(self, x):
        lead, H = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, H)
        T, W, k, El, cap = x2.shape[0], self.W, self.k, self.El, self.cap
        if T > cap:
            raise ValueError(f"{T} tokens exceed the capacity {cap}")
        inds, w = self.route_fn(x2)
        inds = inds.reshape(T, k).to(torch.int64)
        w = w.reshape(T, k)
        slot = plan_slots(inds, El, W)
        # send buffers: [W destinations, cap slots, ...]
        sx = x2.new_zeros((W, cap, H))
        slid = torch.full((W, cap, k), -1, dtype=torch.int64)
        sw = torch.zeros((W, cap, k), dtype=w.dtype)
        stok = torch.zeros((W, cap), dtype=torch.int64)
        count = torch.zeros(W, dtype=torch.int64)
        for d in range(W):
            t = (slot[:, d] >= 0).nonzero().squeeze(-1)
            s = slot[t, d]
            sx[d, s] = x2[t]
            mine = (inds[t] >= d * El) & (inds[t] < (d + 1) * El)
            slid[d, s] = torch.where(mine, inds[t] - d * El, torch.full_like(inds[t], -1))
            sw[d, s] = w[t]
            stok[d, s] = t
            count[d] = t.numel()
        rx, rlid, rw, rtok, rcount = (self._a2a(b) for b in (sx, slid, sw, stok, count))
        live = torch.arange(cap)[None, :] < rcount[:, None]  # [W sources, cap]
        rlid = torch.where(live[..., None], rlid, torch.full_like(rlid, -1))
        y = self.expert_fn(rx.reshape(W * cap, H), rlid.reshape(W * cap, k))
        y = y.reshape(W, cap, k, H).to(torch.float32)
        term = _bf(_bf(y) * rw.to(torch.float32)[..., None])
        # return: for each source, its combine rows [cap tokens, k picks, H]
        back = torch.zeros((W, cap, k, H), dtype=torch.float32)
        ok = rlid >= 0
        for s in range(W):
            tt, jj = ok[s].nonzero(as_tuple=True)
            if tt.numel():
                back[s, rtok[s, tt], jj] = term[s, tt, jj]
        got = self._a2a(back)  # got[d] = the rows owner d computed for this rank's picks
        owner = torch.div(inds, El, rounding_mode="floor")  # [T, k]
        rows = got[owner, torch.arange(T)[:, None], torch.arange(k)[None, :]]  # [T, k, H]
        acc = rows.sum(dim=1) if k else x2.new_zeros((T, H), dtype=torch.float32)
        out = _bf(_bf(acc) * float(self.scale))
        if self.shared_fn is not None:
            out = _bf(out + self.shared_fn(x2).to(torch.float32))
        return out.to(x.dtype).reshape(*lead, H)


def local_switch_glu(sw, lo, hi=None):
    """A SwitchGLU holding experts [lo, hi) of ``sw`` (copied contiguous), or, with ``lo`` a list
    of expert ids, those experts in that order."""
    from .laguna import SwitchGLU, SwitchLinear
    if hi is None:
        idx = torch.tensor(list(lo), dtype=torch.long, device=sw.gate_proj.weight.device)
        take = lambda t: t.index_select(0, idx).contiguous()  # noqa: E731
        n = idx.numel()
    else:
        take = lambda t: t[lo:hi].contiguous()  # noqa: E731
        n = hi - lo

    def cut(p):
        return SwitchLinear(take(p.weight), take(p.scales), take(p.biases), p.group_size, p.bits)

    return SwitchGLU(sw.input_dims, sw.hidden_dims, n, cut(sw.gate_proj), cut(sw.up_proj),
                     cut(sw.down_proj))


def balanced_placement(counts, W):
    """Experts over W ranks, E/W each, balancing the picks: ``counts`` [E] (picks per expert
    on representative traffic, e.g. summed over the ranks of a calibration batch); experts are
    taken busiest first and each goes to the least-loaded rank that still has room (greedy
    longest-processing-time). Returns W lists of expert ids (ascending)."""
    counts = [int(c) for c in counts]
    E = len(counts)
    if E % W:
        raise ValueError(f"{E} experts do not split evenly over {W} ranks")
    El = E // W
    load, held = [0] * W, [[] for _ in range(W)]
    for e in sorted(range(E), key=lambda e: (-counts[e], e)):
        d = min((r for r in range(W) if len(held[r]) < El), key=lambda r: (load[r], r))
        held[d].append(e)
        load[d] += counts[e]
    return [sorted(h) for h in held]


class PeerExpertParallel:
    """Expert-parallel forward of a ``SparseMoeBlock`` over NVLink peer memory.

    Every rank builds one with the same block weights and the same ``capacity`` (tokens per
    rank and forward); the rank keeps its expert slice and maps every peer's arena (CUDA IPC).
    Calls are collective: every rank calls once per forward, in the same order. ``timeout_s``
    bounds each cross-GPU wait; an expired wait leaves NaN outputs and a nonzero ``status()``.
    Outputs equal the one-GPU block's bit for bit when both take the same product path: the
    owners run the tensor-core path when the capacity exceeds LG_MOE_GEMV_MAX_ROWS / (k + 1)
    tokens, as the one-GPU block does for that many tokens.

    ``device_epoch=True``: the forwards' epochs are counted on the device (every call passes
    epoch 0 and ends with ``lg_ep_advance``), so a forward can be captured in a CUDA graph and
    replayed (batched decode steps); ``expert_path`` forces the owners' product path
    (``_lib.LG_PATH_*``) instead of the capacity rule.
    """

    def __init__(self, blk, capacity, group=None, timeout_s=5.0, device_epoch=False,
                 expert_path=None, placement=None):
        from . import _lib, ops
        self.lib = _lib.lib()
        self.blk = blk
        self.group = group
        self.W = W = dist.get_world_size(group)
        self.rank = r = dist.get_rank(group)
        E = blk.num_experts
        if E % W:
            raise ValueError(f"{E} experts do not split evenly over {W} ranks")
        sw = blk.switch_mlp
        self.E, self.El, self.k = E, E // W, blk.top_k
        self.H, self.I = sw.input_dims, sw.hidden_dims
        self.cap, self.timeout = int(capacity), float(timeout_s)
        self.dev = sw.gate_proj.weight.device
        # ``placement``: W lists of expert ids (E/W each, together every expert once; the same
        # on every rank), e.g. ``balanced_placement``; None: rank r holds [r*E/W, (r+1)*E/W)
        self.owner_of = self.local_of = None
        if placement is None:
            self.local = local_switch_glu(sw, r * self.El, (r + 1) * self.El)
        else:
            placement = [list(map(int, p)) for p in placement]
            flat = sorted(e for p in placement for e in p)
            if len(placement) != W or flat != list(range(E)) or \
                    any(len(p) != self.El for p in placement):
                raise ValueError(f"placement must split the {E} experts into {W} lists of "
                                 f"{self.El}")
            owner, local = [0] * E, [0] * E
            for d, p in enumerate(placement):
                for j, e in enumerate(p):
                    owner[e], local[e] = d, j
            self.owner_of = torch.tensor(owner, dtype=torch.int32, device=self.dev)
            self.local_of = torch.tensor(local, dtype=torch.int32, device=self.dev)
            self.local = local_switch_glu(sw, placement[r])
        self.placement = placement
        nb = self.lib.lg_ep_arena_bytes(W, self.cap, self.k, self.H)
        self.arena = torch.zeros(nb, dtype=torch.uint8, device=self.dev)  # flags start at 0
        hb = self.lib.lg_ep_ipc_handle_bytes()
        handle = (ctypes.c_char * hb)()
        off = ctypes.c_size_t(0)
        _lib.call("lg_ep_ipc_handle", self.arena.data_ptr(), ctypes.addressof(handle),
                  ctypes.byref(off))
        mine = (bytes(handle), off.value)
        allh = [None] * W
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        ptrs = []
        for d, (h, o) in enumerate(allh):
            if d == r:
                ptrs.append(self.arena.data_ptr())
                continue
            buf = ctypes.create_string_buffer(h, len(h))
            p, base = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.call("lg_ep_ipc_open", ctypes.addressof(buf), o, ctypes.byref(p),
                      ctypes.byref(base))
            self._opened.append(base.value)
            ptrs.append(p.value)
        self.ptrs = (ctypes.c_void_p * W)(*ptrs)
        sh_off, _ = ctypes.c_size_t(0), None
        cm_off = ctypes.c_size_t(0)
        _lib.call("lg_ep_arena_offsets", W, self.cap, self.k, self.H, ctypes.byref(sh_off),
                  ctypes.byref(cm_off))
        self.shared_rows = self.arena[sh_off.value:sh_off.value + self.cap * self.H * 2] \
            .view(torch.bfloat16).view(self.cap, self.H)
        self.ws_bytes = self.lib.lg_ep_experts_workspace_bytes(W, self.cap, self.H, self.I,
                                                              self.El, self.k)
        self.ws = ops.workspace(self.dev, "ep_moe", self.ws_bytes)
        # the owner's path for the received rows: the same on every rank (by the capacity)
        self.expert_path = _lib.LG_PATH_TENSOR \
            if self.cap * (self.k + 1) > _lib.LG_MOE_GEMV_MAX_ROWS \
            else _lib.LG_PATH_GEMV
        if expert_path is not None:
            self.expert_path = int(expert_path)
        self.device_epoch = bool(device_epoch)
        self.epoch = 0
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=group)  # every peer mapped before anyone writes

    def __call__(self, x):
        from . import _lib, ops
        lead, H = x.shape[:-1], x.shape[-1]
        x2 = ops._c(x.reshape(-1, H), torch.bfloat16)
        T = x2.shape[0]
        if T > self.cap:
            raise ValueError(f"{T} tokens exceed the capacity {self.cap}")
        self.epoch += 1
        ep_arg = 0 if self.device_epoch else self.epoch
        main = torch.cuda.current_stream(self.dev)
        st = main.cuda_stream
        # the product path the one-GPU block takes for these tokens (tensor cores above
        # LG_MOE_GEMV_MAX_ROWS pick rows), so that the outputs equal it bit for bit
        big = T * (self.k + 1) > _lib.LG_MOE_GEMV_MAX_ROWS
        sh = self.blk.shared_expert
        side = None
        if sh is not None and T:
            # the shared expert needs only x: it runs on a second stream beside the routing, the
            # dispatch's peer stores and the owners' wait for the other sources; the combine
            # waits for it
            side = self._side_stream()
            side.wait_stream(main)
            with torch.cuda.stream(side):
                ops.qmlp(x2, sh.mats, path="tensor" if big else "gemv",
                         out=self.shared_rows[:T])
        if T:
            inds, w = self.blk.route(x2)
            inds, w = ops._c(inds, torch.int32), ops._c(w, torch.bfloat16)
        else:  # a rank without tokens still takes part in both exchanges
            inds = torch.empty(0, self.k, dtype=torch.int32, device=self.dev)
            w = torch.empty(0, self.k, dtype=torch.bfloat16, device=self.dev)
        arenas = ctypes.addressof(self.ptrs)
        _lib.call("lg_ep_dispatch_mapped", x2.data_ptr(), inds.data_ptr(), w.data_ptr(), T,
                  self.cap, H, self.k, self.E, self.W, self.rank, arenas, ep_arg,
                  None if self.owner_of is None else self.owner_of.data_ptr(),
                  None if self.local_of is None else self.local_of.data_ptr(), st)
        g, u, d = (ops._qm(m) for m in self.local.mats)
        _lib.call("lg_ep_experts", self.W, self.cap, H, self.I, self.El, self.k,
                  *(t.data_ptr() for t in g), *(t.data_ptr() for t in u),
                  *(t.data_ptr() for t in d), self.rank, arenas, ep_arg, self.timeout,
                  self.expert_path, self.ws.data_ptr(), self.ws_bytes, st)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=self.dev)
        if side is not None:
            main.wait_stream(side)
        _lib.call("lg_ep_combine", inds.data_ptr(), T, self.cap, H, self.k, self.E,
                  float(self.blk.routed_scaling_factor), int(sh is not None), self.W, self.rank,
                  arenas, ep_arg, self.timeout, out.data_ptr(), st)
        if self.device_epoch:
            _lib.call("lg_ep_advance", self.arena.data_ptr(), st)
        return out.reshape(*lead, H)

    def _side_stream(self):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.dev)
        return self._side

    def status(self, reset=True):
        """Status word of this rank's arena: 0, or (code | source << 8) of the first wait that
        expired (code 1: dispatch, 2: combine). Synchronises."""
        from . import _lib
        v = ctypes.c_int(0)
        _lib.call("lg_ep_status", self.arena.data_ptr(), int(bool(reset)), ctypes.byref(v))
        return v.value

    def close(self):
        """Unmap the peers' arenas (after the last forward of every rank)."""
        from . import _lib
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        for base in self._opened:
            _lib.call("lg_ep_ipc_close", base)
        self._opened = []


def bench_block(E, k, H, I, I_sh, zipf, scale, seed=0):
    """The config-5 block: the same seeded weights (Zipf-biased router) on every rank."""
    from . import synth
    blk, _ = synth.moe_block(0, E, k, H, I, I_sh, seed=seed, zipf=zipf,
                             routed_scaling_factor=scale)
    return blk
