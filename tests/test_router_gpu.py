"""Router kernel vs the oracle (laguna_mlx/laguna.py:137-145).

Indices must be bit-exact against the oracle's selection run on the kernel's own logits
(identical logits); rows where the k-th and (k+1)-th biased scores are within 2 ulp are
reported as ties and checked as sets up to the tie. Weights agree to bf16 rounding."""
import pytest
import torch

from oracle import moe_ref
from tests._util import gen, normal

pytestmark = pytest.mark.gpu


def _check(inds, w, logits, bias, k, norm=True, score_fn="sigmoid"):
    lg = logits.cpu()
    scores = torch.sigmoid(lg) if score_fn == "sigmoid" else torch.softmax(lg, -1)
    sel = scores + bias.cpu().float()
    ref = moe_ref.topk_indices(sel, k)
    tie = moe_ref.tie_rows(sel, k)
    got = inds.cpu().long()
    assert torch.equal(got[~tie], ref[~tie])
    for r in tie.nonzero().flatten().tolist():
        kth = torch.sort(sel[r], descending=True).values[k - 1]
        strict = set((sel[r] > kth * (1 + 2 ** -21) + 1e-30).nonzero().flatten().tolist())
        assert strict <= set(got[r].tolist())
    wr = torch.gather(scores, -1, got)
    if norm:
        wr = wr / wr.sum(-1, keepdim=True)
    torch.testing.assert_close(w.cpu().float(), wr, atol=1e-6, rtol=2 ** -7)
    return tie


@pytest.mark.parametrize("T,E,k,H", [(16, 128, 8, 2048), (4096, 128, 8, 2048), (1, 64, 8, 2048),
                                     (10, 8, 2, 64), (33, 256, 16, 128), (7, 40, 5, 192),
                                     (300, 40, 5, 192), (520, 256, 16, 128), (777, 100, 8, 1024)])
def test_router_matches_oracle(T, E, k, H):
    g = gen(T * 1000 + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    W = normal((E, H), 0.02, g)
    bias = normal((E,), 0.01, g)
    from lagunalab_b200 import ops
    inds, w, logits, counts = ops.router_topk(x.cuda(), W.cuda(), bias.cuda(), k, counts=True)
    ref_logits = x.float() @ W.T
    torch.testing.assert_close(logits.cpu(), ref_logits, atol=2e-5, rtol=1e-5)
    _check(inds, w, logits, bias, k)
    # histogram invariants (lagunaLab tests/test_hooks.py:10-22): counts sum to T*k,
    # gate mass sums to T with norm_topk_prob
    c = counts.cpu()
    assert int(c.sum()) == T * k
    assert torch.equal(c, torch.bincount(inds.cpu().reshape(-1).long(), minlength=E).int())
    assert abs(float(w.float().sum()) - T) < 1e-2 * T


def test_router_ties_lower_index_first_and_masked_experts():
    from lagunalab_b200 import ops
    T, E, H, k = 64, 32, 128, 4
    g = gen(7)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    W = normal((E, H), 0.05, g)
    W[5] = W[3]            # identical logits: expert 3 must come before 5
    W[20] = W[3]
    bias = torch.zeros(E)
    bias[::2] = float("-inf")  # pruned experts (bias -> -inf)
    bias[3] = 0.0
    bias[20] = 0.0
    inds, w, logits = ops.router_topk(x.cuda(), W.cuda(), bias.cuda(), k)
    _check(inds, w, logits, bias, k)
    got = inds.cpu()
    masked = set(range(0, E, 2)) - {20}
    assert not (set(got.reshape(-1).tolist()) & masked)
    for r in range(T):
        row = got[r].tolist()
        if 3 in row and 5 in row:
            assert row.index(3) < row.index(5)
        if 3 in row and 20 in row:
            assert row.index(3) < row.index(20)


def test_router_more_picks_than_live_experts():
    from lagunalab_b200 import ops
    E, H, k = 16, 64, 6
    x = torch.randn(3, H, generator=gen(1)).to(torch.bfloat16)
    W = normal((E, H), 0.05, gen(2))
    bias = torch.full((E,), float("-inf"))
    bias[[2, 9, 11]] = 0.0
    inds, w, logits = ops.router_topk(x.cuda(), W.cuda(), bias.cuda(), k)
    got = inds.cpu()
    for r in range(3):
        assert set(got[r, :3].tolist()) == {2, 9, 11}
        assert got[r, 3:].tolist() == [0, 1, 3]   # masked ones: lower index first
    _check(inds, w, logits, bias, k)


def test_router_nan_keys_are_never_picked():
    """A NaN selection key (here through a NaN bias) is out of play: the picks are the top-k
    of the other keys, and past the last of those the picks are -1 with weight 0."""
    from lagunalab_b200 import ops
    T, H = 24, 128
    g = gen(13)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    for E, k, nan_experts in ((32, 8, [1, 6, 17, 30]), (40, 6, list(range(4, 40)))):
        W = normal((E, H), 0.05, g)
        bias = normal((E,), 0.01, g)
        bias[nan_experts] = float("nan")
        inds, w, logits = ops.router_topk(x.cuda(), W.cuda(), bias.cuda(), k)
        sel = torch.sigmoid(logits.cpu()) + bias
        live = [e for e in range(E) if e not in nan_experts]
        ref = moe_ref.topk_indices(sel[:, live], min(k, len(live)))
        ref = torch.tensor(live)[ref]
        got = inds.cpu().long()
        n = ref.shape[1]
        # sets, off rows whose n-th and (n+1)-th live keys are within last-ulp rounding
        tie = moe_ref.tie_rows(sel[:, live], n) if n < len(live) else torch.zeros(T, dtype=bool)
        assert torch.equal(got[~tie, :n].sort(-1).values, ref[~tie].sort(-1).values)
        assert (got[:, n:] == -1).all() and (w.cpu()[:, n:].float() == 0).all()
        assert not set(got.reshape(-1).tolist()) & set(nan_experts)


def test_router_8bit_gate():
    from lagunalab_b200 import ops
    T, E, H, k = 40, 64, 2048, 8
    g = gen(11)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    W = normal((E, H), 0.02, g)
    q = ops.quantize(W.cuda(), 64, 8)
    bias = normal((E,), 0.01, g)
    inds, w, logits = ops.router_topk(x.cuda(), q, bias.cuda(), k)
    ref = moe_ref.router_logits(x, tuple(t.cpu() for t in q))
    # both are bf16-rounded fp32 sums: at most one bf16 ulp apart
    assert ((logits.cpu() - ref).abs() <= ref.abs() * 2 ** -7 + 1e-6).all()
    _check(inds, w, logits, bias, k)


def test_router_softmax_mode_and_no_norm():
    from lagunalab_b200 import ops
    T, E, H, k = 20, 128, 256, 8
    g = gen(5)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    W = normal((E, H), 0.1, g)
    bias = torch.zeros(E)
    inds, w, logits = ops.router_topk(x.cuda(), W.cuda(), bias.cuda(), k, norm_topk_prob=True,
                                      score_fn="softmax")
    _check(inds, w, logits, bias, k, score_fn="softmax")
    inds, w, logits = ops.router_topk(x.cuda(), W.cuda(), bias.cuda(), k, norm_topk_prob=False)
    _check(inds, w, logits, bias, k, norm=False)


def test_plan_is_expert_contiguous_and_ordered():
    from lagunalab_b200 import ops
    T, k, E = 300, 8, 64
    g = gen(3)
    inds = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    counts, offsets, perm = ops.moe_plan(inds.cuda(), E, with_shared=True)
    flat = inds.reshape(-1).long()
    c = torch.bincount(flat, minlength=E)
    assert counts.cpu()[:E].tolist() == c.tolist() and int(counts[E]) == T
    off = offsets.cpu().tolist()
    assert off[0] == 0 and off[E] == T * k and off[E + 1] == T * k + T
    p = perm.cpu().long()
    want = torch.cat([(flat == e).nonzero().flatten() for e in range(E)])
    assert torch.equal(p[:T * k], want)
    assert torch.equal(p[T * k:], torch.arange(T * k, T * k + T))
