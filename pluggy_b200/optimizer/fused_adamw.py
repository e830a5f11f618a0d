"""AdamW whose CUDA step is one sm_100a multi-tensor kernel launch.

Parity: the reference builds ``torch.optim.AdamW(..., fused=True)``
(``pluggy/optimizer/builder.py:20-46``, config ``optimizer.config.fused``).
This class IS a ``torch.optim.AdamW`` (same param groups, same ``state_dict``
keys ``step/exp_avg/exp_avg_sq``), so checkpoints move between the two
frameworks unchanged. Only ``step()`` differs:

* CUDA params: ``pluggy_b200.ops.optim.adamw_step`` updates every param of a
  group in ONE launch (a device table of tensor pointers, grid-stride over
  fixed-size chunks). It optionally multiplies grads by a device-resident clip
  coefficient (so clipping costs no extra pass and no host sync) and can write a
  bf16 copy of each updated param into a registered shadow tensor (the bf16
  weights the GEMMs read), replacing a separate cast pass.
* CPU params: the exact AdamW math in eager torch (oracle / gloo tests).
* CUDA-graph steps (``use_device_hyper``): the kernel reads (lr, bc1, bc2) from a
  per-group device tensor that :meth:`advance` fills on the host before each replay,
  and :meth:`step` (run once, under capture) leaves the step counts to ``advance``.

Math (decoupled weight decay, PyTorch's formulation):
``p -= lr*wd*p; m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*g^2;
p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps)``.
"""

from __future__ import annotations

import math

import torch


class FusedAdamW(torch.optim.AdamW):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2,
                 fused: bool | None = None, foreach: bool | None = None, **kw):
        betas = tuple(betas)
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         foreach=False, fused=False, **kw)
        self.use_kernel = True if fused is None else bool(fused)
        self._grad_scale: torch.Tensor | None = None
        self._shadows: dict[int, torch.Tensor] = {}
        self._hyper: list[torch.Tensor] | None = None

    # ------------------------------------------------------- CUDA-graph steps
    def use_device_hyper(self, device) -> None:
        """Switch to device-resident (lr, bc1, bc2) per param group (see :meth:`advance`).
        Every param must already have its state (run one eager step first)."""
        assert all(len(self.state[p]) > 0 for g in self.param_groups for p in g["params"]), (
            "use_device_hyper: run an eager step first so every param has its AdamW state")
        self._hyper = [torch.zeros(3, dtype=torch.float32, device=device)
                       for _ in self.param_groups]

    @torch.no_grad()
    def advance(self) -> None:
        """The host half of one step in device-hyper mode: count the step and upload
        this step's (lr, bc1, bc2) of each group (a fresh pinned buffer per upload, so an
        upload still queued behind earlier work is never overwritten)."""
        assert self._hyper is not None, "advance() needs use_device_hyper()"
        for group, hyper in zip(self.param_groups, self._hyper, strict=True):
            ps = group["params"]
            if not ps:
                continue
            for p in ps:
                self.state[p]["step"] += 1
            step = float(self.state[ps[0]]["step"])
            b1, b2 = group["betas"]
            lr = group["lr"]
            lr = float(lr) if not torch.is_tensor(lr) else float(lr.item())
            host = torch.tensor([lr, 1 - b1 ** step, 1 - b2 ** step], dtype=torch.float32)
            if hyper.is_cuda:
                hyper.copy_(host.pin_memory(), non_blocking=True)
            else:
                hyper.copy_(host)

    # ------------------------------------------------------------------ hooks
    def set_grad_scale(self, coef: torch.Tensor | None) -> None:
        """Multiply grads by ``coef`` (0-d fp32 device tensor) inside the next step."""
        self._grad_scale = coef

    def register_bf16_shadow(self, param: torch.Tensor, shadow: torch.Tensor) -> None:
        """After each step, write ``param`` cast to bf16 into ``shadow`` (same numel)."""
        assert shadow.numel() == param.numel() and shadow.dtype == torch.bfloat16
        self._shadows[id(param)] = shadow

    def clear_bf16_shadows(self) -> None:
        self._shadows.clear()

    def add_shadow_listener(self, fn) -> None:
        """``fn(params)`` runs after each step with the params whose shadows were written."""
        if not hasattr(self, "_shadow_listeners"):
            self._shadow_listeners = []
        if fn not in self._shadow_listeners:
            self._shadow_listeners.append(fn)

    def _notify_shadows(self, ps) -> None:
        written = [p for p in ps if id(p) in self._shadows]
        if written:
            for fn in getattr(self, "_shadow_listeners", ()):
                fn(written)

    # ------------------------------------------------------------------- step
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        scale = self._grad_scale
        self._grad_scale = None
        if self._hyper is not None:
            return self._step_device_hyper(scale, loss)
        for group in self.param_groups:
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            lr = group["lr"]
            lr = float(lr) if not torch.is_tensor(lr) else float(lr.item())
            b1, b2 = group["betas"]
            wd, eps = group["weight_decay"], group["eps"]
            # lazily create state in the torch.optim.AdamW layout
            for p in params:
                st = self.state[p]
                if len(st) == 0:
                    st["step"] = torch.tensor(0.0, dtype=torch.float32)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            # group params by step count (normally one bucket)
            by_step: dict[float, list] = {}
            for p in params:
                st = self.state[p]
                st["step"] += 1
                by_step.setdefault(float(st["step"]), []).append(p)
            for step, ps in by_step.items():
                bc1 = 1 - b1 ** step
                bc2 = 1 - b2 ** step
                if ps[0].is_cuda and self.use_kernel:
                    from pluggy_b200.ops import optim as _optim

                    _optim.adamw_step(
                        ps, [p.grad for p in ps], [self.state[p]["exp_avg"] for p in ps],
                        [self.state[p]["exp_avg_sq"] for p in ps],
                        [self._shadows.get(id(p)) for p in ps],
                        lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd,
                        bias_correction1=bc1, bias_correction2=bc2, grad_scale=scale)
                    # the kernel wrote through raw pointers: tell autograd (and the bf16
                    # weight caches keyed on the version counter) that params changed
                    torch.autograd.graph.increment_version(ps)
                    self._notify_shadows(ps)
                else:
                    for p in ps:
                        g = p.grad if scale is None else p.grad * scale
                        st = self.state[p]
                        p.mul_(1 - lr * wd)
                        st["exp_avg"].lerp_(g, 1 - b1)
                        st["exp_avg_sq"].mul_(b2).addcmul_(g, g, value=1 - b2)
                        denom = (st["exp_avg_sq"].sqrt() / math.sqrt(bc2)).add_(eps)
                        p.addcdiv_(st["exp_avg"], denom, value=-lr / bc1)
                        sh = self._shadows.get(id(p))
                        if sh is not None:
                            sh.copy_(p.view_as(sh))
                    self._notify_shadows(ps)
        return loss

    def _step_device_hyper(self, scale, loss):
        from pluggy_b200.ops import optim as _optim

        for group, hyper in zip(self.param_groups, self._hyper, strict=True):
            ps = [p for p in group["params"] if p.grad is not None]
            if not ps:
                continue
            assert ps[0].is_cuda and self.use_kernel, "device-hyper steps run the CUDA kernel"
            b1, b2 = group["betas"]
            _optim.adamw_step(
                ps, [p.grad for p in ps], [self.state[p]["exp_avg"] for p in ps],
                [self.state[p]["exp_avg_sq"] for p in ps], [self._shadows.get(id(p)) for p in ps],
                lr=0.0, beta1=b1, beta2=b2, eps=group["eps"], weight_decay=group["weight_decay"],
                bias_correction1=1.0, bias_correction2=1.0, grad_scale=scale, hyper=hyper)
            torch.autograd.graph.increment_version(ps)
            self._notify_shadows(ps)
        return loss
