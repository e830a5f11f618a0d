"""Differentiable linear layer on the tcgen05 GEMM (bf16 compute, fp32 master weight).

``linear(x, weight, weight_lowp=None)`` computes ``x W^T`` in bf16 with fp32
accumulation; its backward produces ``dx`` (bf16, dgrad GEMM) and ``dW`` in fp32
straight from the wgrad GEMM's accumulator (no bf16 round trip of the weight
gradient, which the reference's autocast path has). ``weight_lowp`` is an
optional cached bf16 copy of ``weight`` (see :class:`WeightCache`).
"""

from __future__ import annotations

import torch

from pluggy_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad


class WeightCache:
    """bf16 copies of fp32 parameters, refreshed when the parameter changes.

    Keyed on the parameter object; a copy is recast whenever the parameter's
    version counter moved (optimizer step, load_state_dict, manual edits), so
    forward passes within one optimizer step share one cast.

    ``bind_optimizer(opt)`` (an optimizer with bf16 shadows, e.g.
    :class:`~pluggy_b200.optimizer.fused_adamw.FusedAdamW`) removes even that
    cast: every cached copy is registered as the parameter's shadow, the optimizer
    writes the bf16 value in the same kernel that updates the fp32 master, and
    tells the cache the copy is current.
    """

    def __init__(self):
        self._store: dict = {}
        self._params: dict[int, torch.Tensor] = {}
        self._cat_params: dict[str, list[torch.Tensor]] = {}
        self._opt = None
        # set by FSDP2: a gather rewrites the full parameter's storage without moving
        # its version counter, so every get() recasts (into the same bf16 buffer)
        self.always_recast = False
        # set by FSDP2's low-precision gathers: ``provider(params)`` returns the bf16
        # weights already gathered in place (or None), read instead of a cached copy
        self.provider = None

    def bind_optimizer(self, opt) -> None:
        if self._opt is opt:
            return
        self._opt = opt
        opt.add_shadow_listener(self._shadows_written)
        for key, (_, _, lp) in list(self._store.items()):
            self._register(key, lp)

    def _register(self, key, lp: torch.Tensor) -> None:
        if isinstance(key, str):
            off = 0
            for p in self._cat_params[key]:
                n = p.shape[0]
                self._opt.register_bf16_shadow(p, lp[off:off + n])
                off += n
        else:
            p = self._params.get(key)
            if p is not None:
                self._opt.register_bf16_shadow(p, lp)

    def _shadows_written(self, params: list[torch.Tensor]) -> None:
        ids = {id(p) for p in params}
        for p in params:
            hit = self._store.get(id(p))
            if hit is not None:
                self._store[id(p)] = (p._version, p.data_ptr(), hit[2])
        for key, ps in self._cat_params.items():
            hit = self._store.get(key)
            if hit is not None and any(id(p) in ids for p in ps):
                self._store[key] = (tuple((p._version, p.data_ptr()) for p in ps), None, hit[2])

    def get(self, p: torch.Tensor) -> torch.Tensor:
        if self.provider is not None:
            v = self.provider([p])
            if v is not None:
                return v
        key = id(p)
        ver = p._version
        hit = self._store.get(key)
        if hit is not None and hit[0] == ver and hit[1] == p.data_ptr() and not self.always_recast:
            return hit[2]
        from pluggy_b200.ops._ext import ext

        lp = hit[2] if hit is not None and hit[2].shape == p.shape else torch.empty(
            p.shape, dtype=torch.bfloat16, device=p.device)
        if p.is_cuda:
            ext().cast_f32_bf16(p.detach().contiguous(), lp)
        else:
            lp.copy_(p.detach())
        self._store[key] = (ver, p.data_ptr(), lp)
        self._params[key] = p
        if self._opt is not None and hit is None:
            self._register(key, lp)
        return lp

    def get_cat(self, params: list[torch.Tensor], key: str) -> torch.Tensor:
        """bf16 concatenation (dim 0) of several params, cached as one buffer."""
        if self.provider is not None:
            v = self.provider(list(params))
            if v is not None:
                return v
        vers = tuple((p._version, p.data_ptr()) for p in params)
        hit = self._store.get(key)
        if hit is not None and hit[0] == vers and not self.always_recast:
            return hit[2]
        from pluggy_b200.ops._ext import ext

        rows = sum(p.shape[0] for p in params)
        lp = hit[2] if hit is not None else torch.empty(
            (rows, *params[0].shape[1:]), dtype=torch.bfloat16, device=params[0].device)
        off = 0
        for p in params:
            n = p.shape[0]
            if p.is_cuda:
                ext().cast_f32_bf16(p.detach().contiguous(), lp[off:off + n])
            else:
                lp[off:off + n].copy_(p.detach())
            off += n
        self._store[key] = (vers, None, lp)
        self._cat_params[key] = list(params)
        if self._opt is not None and hit is None:
            self._register(key, lp)
        return lp

    def clear(self) -> None:
        self._store.clear()
        self._cat_params.clear()
        self._params.clear()
        if self._opt is not None:
            self._opt.clear_bf16_shadows()


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, w_lowp):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).to(torch.bfloat16).contiguous()
        w = w_lowp if w_lowp is not None else weight.to(torch.bfloat16)
        y = linear_fwd(x2, w)
        ctx.save_for_backward(x2, w)
        ctx.x_dtype = x.dtype
        ctx.shp = shp
        return y.reshape(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = linear_dgrad(dy2, w).reshape(ctx.shp).to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            dw = linear_wgrad(dy2, x2)
        return dx, dw, None


def linear(x: torch.Tensor, weight: torch.Tensor, weight_lowp: torch.Tensor | None = None):
    if x.is_cuda:
        return _Linear.apply(x, weight, weight_lowp)
    return torch.nn.functional.linear(x, weight.to(x.dtype))
