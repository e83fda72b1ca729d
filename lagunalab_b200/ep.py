"""Expert parallelism for the MoE block over torch.distributed (NCCL on B200, gloo in tests).

Rank r of W owns the contiguous experts [r*E/W, (r+1)*E/W); router and shared expert are
replicated and every rank routes its own tokens. One forward:

1. route locally (the fused router kernel): inds [T, k], w [T, k];
2. order the T*k picks by destination rank (stable, so picks keep token order inside a
   destination), exchange per-destination counts (all-to-all of W ints);
3. dispatch: all-to-all of the picked token rows (bf16 [*, H]) and their local expert ids;
4. local experts: SwitchGLU over the received rows (k = 1 per row, the grouped kernels);
5. combine: all-to-all of the expert outputs back to the source rank, un-permute, then
   out = sum_k w * y * routed_scale + shared(x).

Every rank takes the same collective steps in the same order. The compute steps are
injectable (``route_fn``, ``expert_fn``, ``shared_fn``) so the control flow can be tested on
CPU ranks with the oracle.
"""
import torch
import torch.distributed as dist


class ExpertParallelMoE:
    def __init__(self, E, k, routed_scaling_factor, route_fn, expert_fn, shared_fn=None,
                 group=None):
        self.group = group
        self.W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.W:
            raise ValueError(f"{E} experts do not split evenly over {self.W} ranks")
        self.E, self.k, self.El = E, k, E // self.W
        self.scale = routed_scaling_factor
        self.route_fn, self.expert_fn, self.shared_fn = route_fn, expert_fn, shared_fn

    def dispatch(self, x, inds):
        """Returns (recv_rows, recv_local_ids, order, send_counts, recv_counts)."""
        T, k = inds.shape
        flat = inds.reshape(-1).to(torch.int64)
        dest = torch.div(flat, self.El, rounding_mode="floor")
        order = torch.sort(dest, stable=True).indices
        send_counts = torch.bincount(dest, minlength=self.W).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        rows = x[torch.div(order, k, rounding_mode="floor")].contiguous()
        lid = (flat[order] - dest[order] * self.El).to(torch.int32).contiguous()
        recv_rows = rows.new_empty((sum(rc), x.shape[-1]))
        recv_lid = lid.new_empty((sum(rc),))
        dist.all_to_all_single(recv_rows, rows, rc, sc, group=self.group)
        dist.all_to_all_single(recv_lid, lid, rc, sc, group=self.group)
        return recv_rows, recv_lid, order, sc, rc

    def combine(self, y_recv, order, sc, rc, shape):
        """Send expert outputs back and restore pick order -> [T, k, H]."""
        T, k, H = shape
        y_back = y_recv.new_empty((sum(sc), H))
        dist.all_to_all_single(y_back, y_recv.contiguous(), sc, rc, group=self.group)
        y = torch.empty_like(y_back)
        y[order] = y_back
        return y.view(T, k, H)

    def __call__(self, x):
        lead = x.shape[:-1]
        H = x.shape[-1]
        x2 = x.reshape(-1, H)
        inds, w = self.route_fn(x2)
        inds = inds.reshape(-1, self.k)
        w = w.reshape(-1, self.k)
        recv_rows, recv_lid, order, sc, rc = self.dispatch(x2, inds)
        # expert outputs travel in the input's dtype on every rank (a rank that received no
        # rows must post a combine exchange of the same element size as the others)
        if recv_rows.shape[0]:
            y_recv = self.expert_fn(recv_rows, recv_lid).to(x2.dtype)
        else:
            y_recv = recv_rows.new_empty((0, H))
        y = self.combine(y_recv, order, sc, rc, (x2.shape[0], self.k, H))
        out = (y.float() * w.float().unsqueeze(-1)).sum(1) * self.scale
        if self.shared_fn is not None:
            out = out + self.shared_fn(x2).float()
        return out.to(x.dtype).reshape(*lead, H)


def local_switch_glu(sw, lo, hi):
    """A SwitchGLU view holding experts [lo, hi) of ``sw`` (copied contiguous)."""
    from .laguna import SwitchGLU, SwitchLinear

    def cut(p):
        return SwitchLinear(p.weight[lo:hi].contiguous(), p.scales[lo:hi].contiguous(),
                            p.biases[lo:hi].contiguous(), p.group_size, p.bits)

    return SwitchGLU(sw.input_dims, sw.hidden_dims, hi - lo, cut(sw.gate_proj),
                     cut(sw.up_proj), cut(sw.down_proj))


def from_block(blk, group=None):
    """Expert-parallel forward for a SparseMoeBlock: this rank keeps its expert slice."""
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    El = blk.num_experts // W
    local = local_switch_glu(blk.switch_mlp, r * El, (r + 1) * El)

    def expert_fn(rows, lid):
        return local(rows, lid.view(-1, 1)).view(-1, rows.shape[-1])

    shared = blk.shared_expert
    return ExpertParallelMoE(blk.num_experts, blk.top_k, blk.routed_scaling_factor, blk.route,
                             expert_fn, shared if shared is not None else None, group), local


def bench_block(T, E, k, H, I, I_sh, zipf, scale, ws, rank):
    """Synthetic config-5 block: same weights on every rank (seed 0), rank-specific tokens;
    each rank keeps only its experts."""
    from . import synth
    blk, _ = synth.moe_block(0, E, k, H, I, I_sh, seed=0, zipf=zipf, routed_scaling_factor=scale)
    fwd, local = from_block(blk)
    blk.switch_mlp = local   # drop the other ranks' experts
    torch.cuda.empty_cache()
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + rank)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    return blk, x, fwd
