"""RoutingRecorder (laguna_mlx/hooks.py:6-48 surface) on CPU tensors: the invariants of
lagunaLab's tests/test_hooks.py:10-22 (counts sum to T*k, mass to T for renormalised weights),
the token mask, and the wrap/unwrap contract on ``route``."""
import numpy as np
import torch

from lagunalab_b200.hooks import RoutingRecorder


class _Args:
    num_experts = 8


class _Moe:
    def __init__(self, seed):
        self.seed = seed

    def route(self, x):
        T = x.shape[0] * x.shape[1]
        g = torch.Generator().manual_seed(self.seed + T)
        s = torch.rand(T, 8, generator=g)
        inds = torch.topk(s, 2, dim=-1).indices.to(torch.int32)
        w = torch.gather(s, -1, inds.long())
        w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
        return inds.view(*x.shape[:2], 2), w.view(*x.shape[:2], 2)


class _Layer:
    def __init__(self, mlp):
        self.mlp = mlp


class _Model:
    args = _Args()

    def __init__(self):
        self.layers = [_Layer(object()), _Layer(_Moe(1)), _Layer(_Moe(2))]

    def __call__(self, x):
        for l in self.layers:
            if hasattr(l.mlp, "route"):
                l.mlp.route(x)


def test_counts_and_mass_invariants():
    m = _Model()
    x = torch.zeros(1, 12, 4)
    with RoutingRecorder(m) as rec:
        m(x)
        m(x)
    assert set(rec.counts) == {1, 2}
    for i in (1, 2):
        assert rec.counts[i].dtype == np.int64 and rec.counts[i].sum() == 2 * 12 * 2
        assert abs(rec.mass[i].sum() - 2 * 12) < 0.05  # bf16 weights renormalised per token
        want = np.zeros(8, np.int64)
        inds, _ = m.layers[i].mlp.route(x)
        np.add.at(want, inds.reshape(-1).numpy(), 2)
        assert (rec.counts[i] == want).all()
    assert "route" not in m.layers[1].mlp.__dict__  # unwrapped on exit


def test_token_mask_counts_only_selected_tokens():
    m = _Model()
    x = torch.zeros(1, 10, 4)
    with RoutingRecorder(m) as rec:
        rec.token_mask = np.arange(10) % 2 == 0
        m(x)
    inds, w = m.layers[1].mlp.route(x)
    keep = inds.reshape(-1, 2)[::2].reshape(-1).numpy()
    want = np.bincount(keep, minlength=8)
    assert (rec.counts[1] == want).all()
    ww = w.reshape(-1, 2)[::2].float().reshape(-1).numpy()
    assert np.allclose(rec.mass[1], np.bincount(keep, weights=ww, minlength=8))
