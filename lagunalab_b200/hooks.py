"""Opt-in routing instrumentation with the surface of laguna_mlx/hooks.py:6-48.

    with RoutingRecorder(model) as rec:
        model(ids)
    rec.counts[layer]  # int64[num_experts]
    rec.mass[layer]    # float64[num_experts], summed routing weights

``rec.token_mask`` (bool over the B*L tokens of the next forwards) restricts counting to some
tokens. Unlike the reference, which copies every layer's routing to numpy (a host sync per
layer), the recorder accumulates on the device: each wrapped ``route`` adds its picks and
weights into per-layer [E] accumulators with two scatter-adds on the model's stream, so a
recorded forward runs without host round trips. ``counts`` and ``mass`` copy all layers to the
host in one transfer when they are read. Weight sums are float64 over bf16 weights, exact in
any addition order, so the totals do not depend on scheduling.
"""
import numpy as np
import torch


class RoutingRecorder:
    def __init__(self, model):
        self.moe = {i: l.mlp for i, l in enumerate(model.layers) if hasattr(l.mlp, "route")}
        self.E = model.args.num_experts
        self.token_mask = None
        self._slot = {layer: j for j, layer in enumerate(self.moe)}
        self._dev = None
        self._host = None
        self._mask_src = self._mask_dev = None

    # accumulators -------------------------------------------------------------------------
    def _acc(self, device):
        if self._dev is None:
            n = len(self.moe)
            self._dev = (torch.zeros(n, self.E, dtype=torch.int64, device=device),
                         torch.zeros(n, self.E, dtype=torch.float64, device=device))
        return self._dev

    def _pull(self):
        if self._host is None:
            if self._dev is None:
                z = np.zeros(self.E, np.int64)
                self._host = ({i: z.copy() for i in self.moe},
                              {i: z.astype(np.float64) for i in self.moe})
            else:
                both = torch.cat([self._dev[0].to(torch.float64), self._dev[1]], 0).cpu().numpy()
                n = len(self.moe)
                self._host = ({i: both[j].astype(np.int64) for i, j in self._slot.items()},
                              {i: both[n + j] for i, j in self._slot.items()})
        return self._host

    @property
    def counts(self):
        return self._pull()[0]

    @property
    def mass(self):
        return self._pull()[1]

    def _mask(self, device):
        m = self.token_mask
        if m is None:
            return None
        if m is not self._mask_src:
            self._mask_src = m
            self._mask_dev = torch.as_tensor(np.asarray(m, dtype=bool)).to(device)
        return self._mask_dev

    # wrapping -----------------------------------------------------------------------------
    def __enter__(self):
        for i, mlp in self.moe.items():
            mlp.route = self._wrap(i, mlp)
        return self

    def __exit__(self, *exc):
        for mlp in self.moe.values():
            del mlp.route

    def _wrap(self, i, mlp):
        orig = type(mlp).route
        slot = self._slot[i]

        def route(x):
            inds, w = orig(mlp, x)
            k = inds.shape[-1]
            flat = inds.reshape(-1).to(torch.int64)
            ww = w.reshape(-1).to(torch.float64)
            one = torch.ones_like(flat)
            m = self._mask(inds.device)
            if m is not None:  # masked-out tokens add zero (no data-dependent shapes, no sync)
                keep = m.reshape(-1, 1).expand(-1, k).reshape(-1)
                one = one * keep
                ww = ww * keep
            counts, mass = self._acc(inds.device)
            counts[slot].index_add_(0, flat, one)
            mass[slot].index_add_(0, flat, ww)
            self._host = None
            return inds, w

        return route
