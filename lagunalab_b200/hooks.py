"""Opt-in routing instrumentation (laguna_mlx/hooks.py:6-48) for the B200 model.

    with RoutingRecorder(model) as rec:
        model(ids)
    rec.counts[layer]  # int64[num_experts]
    rec.mass[layer]    # float64[num_experts], summed routing weights

Recording copies the routing of every MoE layer to the host, so it synchronises per layer;
never leave it on for timing runs.
"""
import numpy as np
import torch


class RoutingRecorder:
    def __init__(self, model):
        self.moe = {i: l.mlp for i, l in enumerate(model.layers) if hasattr(l.mlp, "route")}
        E = model.args.num_experts
        self.counts = {i: np.zeros(E, np.int64) for i in self.moe}
        self.mass = {i: np.zeros(E, np.float64) for i in self.moe}
        self.token_mask = None

    def __enter__(self):
        for i, mlp in self.moe.items():
            mlp.route = self._wrap(i, mlp)
        return self

    def __exit__(self, *exc):
        for mlp in self.moe.values():
            del mlp.route

    def _wrap(self, i, mlp):
        orig = type(mlp).route

        def route(x):
            inds, w = orig(mlp, x)
            k = inds.shape[-1]
            ii = inds.reshape(-1, k).cpu().numpy()
            ww = w.to(torch.float32).reshape(-1, k).cpu().numpy()
            if self.token_mask is not None:
                ii, ww = ii[self.token_mask], ww[self.token_mask]
            np.add.at(self.counts[i], ii.ravel(), 1)
            np.add.at(self.mass[i], ii.ravel(), ww.ravel())
            return inds, w

        return route
